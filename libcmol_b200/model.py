"""ctypes mirror of the libcmol public API (cmol.h + cmol_cuda.h).

Names and argument meanings follow include/cmol.h of the reference
(cmol_load / cmol_session_acquire / cmol_generate / ...); errors raise
CmolError carrying the cmol_err_t code.  Everything runs in libcmol.so.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import CmolError, lib

CMOL_OK, CMOL_ERR_OOM, CMOL_ERR_IO, CMOL_ERR_INVALID, CMOL_ERR_UNSUPPORTED = 0, -1, -2, -3, -4
CMOL_ERR_NO_SESSION, CMOL_ERR_ARGS, CMOL_ERR_CTX_FULL, CMOL_ERR_TRUNC = -5, -6, -7, -8

_vp = C.c_void_p
_ip = C.POINTER(C.c_int32)
_fp = C.POINTER(C.c_float)

LOG_FN = C.CFUNCTYPE(None, C.c_int, C.c_char_p, C.c_void_p)
TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_char_p, C.c_size_t, C.c_int, C.c_void_p)
ID_CB = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_int, C.c_void_p)


class Config(C.Structure):
    """cmol_config_t (include/cmol.h:93-99 of the reference)."""
    _fields_ = [("max_ctx", C.c_int), ("max_sessions", C.c_int), ("prefill_chunk", C.c_int),
                ("log_fn", _vp), ("log_ud", _vp)]


class GenParams(C.Structure):
    """cmol_gen_params_t (include/cmol.h:110-120 of the reference)."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("max_new_tokens", C.c_int), ("seed", C.c_uint),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_int)]

    @classmethod
    def default(cls):
        # CMOL_DEFAULT_PARAMS (include/cmol.h:122-125)
        return cls(0.8, 0.95, 40, 256, 0, 1.1, 64)

    @classmethod
    def make(cls, temperature=0.0, top_p=0.95, top_k=40, max_new_tokens=256, seed=1,
             repeat_penalty=1.0, repeat_last_n=64):
        return cls(temperature, top_p, top_k, max_new_tokens, seed, repeat_penalty, repeat_last_n)


class CudaOptions(C.Structure):
    _fields_ = [("kv_page_tokens", C.c_int), ("kv_pool_frac", C.c_float),
                ("max_batch", C.c_int), ("use_graphs", C.c_int), ("kv_dtype", C.c_int)]


class CudaStats(C.Structure):
    _fields_ = [("decode_steps", C.c_longlong), ("decode_tokens", C.c_longlong),
                ("prefill_tokens", C.c_longlong), ("decode_ms", C.c_double),
                ("step_ms_last", C.c_double), ("weight_bytes", C.c_longlong),
                ("kv_bytes_read", C.c_longlong), ("kernel_launches_per_step", C.c_int),
                ("graph_steps", C.c_int), ("steps", C.c_longlong), ("step_ms_total", C.c_double),
                ("last_fault_code", C.c_uint), ("h2d_bytes_per_step", C.c_longlong),
                ("d2h_bytes_per_step", C.c_longlong)]


class BatchItem(C.Structure):
    _fields_ = [("session", _vp), ("prompt", _ip), ("n_prompt", C.c_int),
                ("params", C.POINTER(GenParams)), ("out", _ip), ("out_cap", C.c_int),
                ("n_out", C.c_int), ("status", C.c_int)]


_declared = False


def api():
    global _declared
    L = lib()
    if _declared:
        return L

    def sig(name, res, args):
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args

    sig("cmol_load", _vp, [C.c_char_p, C.POINTER(Config), C.POINTER(C.c_int)])
    sig("cmol_free", None, [_vp])
    sig("cmol_session_acquire", _vp, [_vp])
    sig("cmol_session_release", None, [_vp])
    sig("cmol_session_reset", None, [_vp])
    sig("cmol_generate", C.c_int, [_vp, C.c_char_p, C.POINTER(GenParams), TOKEN_CB, _vp])
    sig("cmol_encode", C.c_int, [_vp, C.c_char_p, _ip, C.c_int])
    sig("cmol_decode_token", C.c_char_p, [_vp, C.c_int32])
    sig("cmol_strerror", C.c_char_p, [C.c_int])
    sig("cmol_version", C.c_char_p, [])
    sig("cmol_arena_estimate", C.c_size_t, [C.c_char_p, C.POINTER(Config)])
    sig("cmol_format_chatml", C.c_int, [C.c_char_p, C.c_char_p, C.c_char_p, C.c_size_t])
    sig("cmol_format_chatml_turn", C.c_int, [C.c_char_p, C.c_char_p, C.c_size_t])
    sig("cmol_cuda_set_devices", C.c_int, [C.POINTER(C.c_int), C.c_int])
    sig("cmol_cuda_set_options", None, [C.POINTER(CudaOptions)])
    sig("cmol_generate_ids", C.c_int, [_vp, _ip, C.c_int, C.POINTER(GenParams), ID_CB, _vp])
    sig("cmol_generate_batch", C.c_int, [C.POINTER(BatchItem), C.c_int])
    sig("cmol_forward_logits", C.c_int, [_vp, C.c_int32, _fp])
    sig("cmol_forward_logits_batch", C.c_int, [C.POINTER(_vp), _ip, C.c_int, _fp])
    sig("cmol_cuda_debug_inject", C.c_int, [_vp, C.c_int, C.c_int])
    sig("cmol_cuda_kernel_sweep", C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double),
                                            C.POINTER(C.c_longlong), C.POINTER(C.c_double), C.POINTER(C.c_int)])
    sig("cmol_session_n_tokens", C.c_int, [_vp])
    sig("cmol_session_device", C.c_int, [_vp])
    sig("cmol_cuda_session_save", C.c_int, [_vp, _vp, C.c_size_t, C.POINTER(C.c_size_t)])
    sig("cmol_cuda_session_restore", C.c_int, [_vp, _vp, C.c_size_t])
    sig("cmol_vocab_size", C.c_int, [_vp])
    sig("cmol_eos_id", C.c_int, [_vp])
    sig("cmol_cuda_stats", C.c_int, [_vp, C.c_int, C.POINTER(CudaStats)])
    sig("cmol_cuda_stats_reset", None, [_vp])
    sig("cmol_cuda_n_gpus", C.c_int, [_vp])
    sig("cmol_cuda_gemv_sweep", C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(C.c_double),
                                          C.POINTER(C.c_longlong), C.POINTER(C.c_int)])
    _declared = True
    return L


def strerror(code: int) -> str:
    return api().cmol_strerror(code).decode("utf-8", "replace")


def _chk(rc: int, what: str):
    if rc != CMOL_OK:
        raise CmolError(f"{what}: {strerror(rc)} ({rc})")


class Model:
    """cmol_load / cmol_free around one GGUF file."""

    def __init__(self, path: str, max_ctx: int = 2048, max_sessions: int = 4, devices=None,
                 page_tokens: int = 0, max_batch: int = 0, use_graphs: bool = True, log=None,
                 kv_dtype: int = 0):
        L = api()
        if devices is not None:
            arr = (C.c_int * len(devices))(*devices)
            _chk(L.cmol_cuda_set_devices(arr, len(devices)), "cmol_cuda_set_devices")
        opt = CudaOptions(page_tokens, 0.0, max_batch, 1 if use_graphs else 0, kv_dtype)
        L.cmol_cuda_set_options(C.byref(opt))
        self._log_cb = LOG_FN(lambda lvl, msg, ud: log(lvl, msg.decode())) if log else None
        cfg = Config(max_ctx, max_sessions, 512,
                     C.cast(self._log_cb, _vp) if self._log_cb else None, None)
        err = C.c_int(0)
        self.h = L.cmol_load(path.encode(), C.byref(cfg), C.byref(err))
        if not self.h:
            raise CmolError(f"cmol_load: {strerror(err.value)} ({err.value})")
        self.vocab = L.cmol_vocab_size(self.h)
        self.eos = L.cmol_eos_id(self.h)
        self.n_gpus = L.cmol_cuda_n_gpus(self.h)

    def close(self):
        if getattr(self, "h", None):
            api().cmol_free(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def acquire(self):
        s = api().cmol_session_acquire(self.h)
        return Session(self, s) if s else None

    def stats(self, gpu: int = 0) -> CudaStats:
        st = CudaStats()
        _chk(api().cmol_cuda_stats(self.h, gpu, C.byref(st)), "cmol_cuda_stats")
        return st

    def reset_stats(self):
        api().cmol_cuda_stats_reset(self.h)

    def gemv_sweep(self, gpu: int = 0, reps: int = 20):
        """(ms per pass, bytes per pass, launches per pass) of cmol_cuda_gemv_sweep."""
        ms, nb, nl = C.c_double(0), C.c_longlong(0), C.c_int(0)
        _chk(api().cmol_cuda_gemv_sweep(self.h, gpu, reps, C.byref(ms), C.byref(nb), C.byref(nl)),
             "cmol_cuda_gemv_sweep")
        return ms.value, nb.value, nl.value

    def kernel_sweep(self, what: int, gpu: int = 0, reps: int = 10):
        """cmol_cuda_kernel_sweep of the last step: what 0 = weight products,
        1 = attention.  Returns (ms, bytes, flops, launches) per pass."""
        ms, nb, fl, nl = C.c_double(0), C.c_longlong(0), C.c_double(0), C.c_int(0)
        _chk(api().cmol_cuda_kernel_sweep(self.h, gpu, what, reps, C.byref(ms), C.byref(nb), C.byref(fl),
                                          C.byref(nl)), "cmol_cuda_kernel_sweep")
        return ms.value, nb.value, fl.value, nl.value

    def forward_logits_batch(self, sessions, tokens) -> np.ndarray:
        """cmol_forward_logits_batch: one step, one column per session;
        returns the logits [n][vocab]."""
        n = len(sessions)
        hs = (_vp * n)(*[s.h for s in sessions])
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros((n, self.vocab), np.float32)
        _chk(api().cmol_forward_logits_batch(hs, toks.ctypes.data_as(_ip), n, out.ctypes.data_as(_fp)),
             "cmol_forward_logits_batch")
        return out

    def debug_inject(self, kind: int, gpu: int = 0):
        """cmol_cuda_debug_inject: plant a caught error in the next step."""
        _chk(api().cmol_cuda_debug_inject(self.h, gpu, kind), "cmol_cuda_debug_inject")

    def encode(self, text: str, cap: int = 4096):
        out = np.zeros(cap, np.int32)
        n = api().cmol_encode(self.h, text.encode(), out.ctypes.data_as(_ip), cap)
        if n < 0:
            raise CmolError(f"cmol_encode: {strerror(n)}")
        return out[:n]

    def decode_token(self, tid: int):
        r = api().cmol_decode_token(self.h, tid)
        return r

    def generate_batch(self, sessions, prompts, params, out_cap: int = 4096):
        """cmol_generate_batch: all sessions at once; returns list of id arrays."""
        n = len(sessions)
        items = (BatchItem * n)()
        keep = []
        outs = []
        for i, (s, p, pr) in enumerate(zip(sessions, prompts, params)):
            pa = np.ascontiguousarray(p, np.int32)
            o = np.zeros(out_cap, np.int32)
            pp = GenParams(*[getattr(pr, f) for f, _ in GenParams._fields_])
            keep += [pa, pp]
            outs.append(o)
            items[i] = BatchItem(s.h, pa.ctypes.data_as(_ip), len(pa), C.pointer(pp),
                                 o.ctypes.data_as(_ip), out_cap, 0, 0)
        rc = api().cmol_generate_batch(items, n)
        res = [outs[i][:items[i].n_out] for i in range(n)]
        st = [items[i].status for i in range(n)]
        if rc != CMOL_OK:
            raise CmolError(f"cmol_generate_batch: {strerror(rc)} statuses={st}")
        return res


class Session:
    def __init__(self, model: Model, h):
        self.m = model
        self.h = h

    def release(self):
        if self.h:
            api().cmol_session_release(self.h)
            self.h = None

    def reset(self):
        api().cmol_session_reset(self.h)

    @property
    def n_tokens(self) -> int:
        return api().cmol_session_n_tokens(self.h)

    @property
    def device(self) -> int:
        return api().cmol_session_device(self.h)

    def save(self) -> bytes:
        """cmol_cuda_session_save: the session's KV snapshot."""
        n = C.c_size_t(0)
        _chk(api().cmol_cuda_session_save(self.h, None, 0, C.byref(n)), "cmol_cuda_session_save")
        buf = C.create_string_buffer(n.value)
        _chk(api().cmol_cuda_session_save(self.h, buf, n.value, C.byref(n)), "cmol_cuda_session_save")
        return buf.raw

    def restore(self, snap: bytes):
        """cmol_cuda_session_restore: continue from a saved context."""
        _chk(api().cmol_cuda_session_restore(self.h, snap, len(snap)), "cmol_cuda_session_restore")

    def forward_logits(self, token: int) -> np.ndarray:
        out = np.zeros(self.m.vocab, np.float32)
        _chk(api().cmol_forward_logits(self.h, int(token), out.ctypes.data_as(_fp)), "cmol_forward_logits")
        return out

    def generate_ids(self, prompt, params: GenParams, on_token=None):
        """cmol_generate_ids; returns (status, ids).  on_token(id, is_eos) -> int."""
        ids = []

        def cb(t, eos, ud):
            ids.append(int(t))
            return int(on_token(int(t), int(eos))) if on_token else 0

        cfun = ID_CB(cb)
        pa = np.ascontiguousarray(prompt, np.int32)
        rc = api().cmol_generate_ids(self.h, pa.ctypes.data_as(_ip), len(pa), C.byref(params), cfun, None)
        return rc, ids

    def generate(self, text: str, params: GenParams, on_piece=None):
        pieces = []

        def cb(piece, n, eos, ud):
            b = C.string_at(piece, n) if n else b""
            pieces.append((b, int(eos)))
            return int(on_piece(b, int(eos))) if on_piece else 0

        cfun = TOKEN_CB(cb)
        rc = api().cmol_generate(self.h, text.encode(), C.byref(params), cfun, None)
        return rc, pieces
