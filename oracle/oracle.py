"""ctypes bindings for the test-only checkers.

TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke check in
__graft_entry__.py and by bench.py's cpu_baseline / reference legs — never
by the product (libcmol_b200/).

* ``Oracle`` wraps oracle/_build/liborc.so, the C restatement in
  cmol_oracle.c.
* ``Reference`` wraps oracle/_ref/libcmolref.so, the unmodified reference
  (nvlass/libcmol src/cmol.c) compiled from its own sources plus
  ref_driver.c.  It exists wherever ``make -C oracle ref`` ran with the
  reference sources present; on a machine without them it may still travel
  as a prebuilt file.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_SO = os.path.join(HERE, "_build", "liborc.so")
REF_SO = os.path.join(HERE, "_ref", "libcmolref.so")

_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int32)
_u64p = C.POINTER(C.c_uint64)


def fptr(a):
    return a.ctypes.data_as(_fp)


def iptr(a):
    return a.ctypes.data_as(_ip)


class GenParams(C.Structure):
    """Layout of cmol_gen_params_t (include/cmol.h:110-120 of the reference)."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("max_new_tokens", C.c_int), ("seed", C.c_uint),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_int)]

    @classmethod
    def make(cls, temperature=0.0, top_p=0.95, top_k=40, max_new_tokens=256, seed=1,
             repeat_penalty=1.0, repeat_last_n=64):
        return cls(temperature, top_p, top_k, max_new_tokens, seed, repeat_penalty, repeat_last_n)


class OrcTensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int)]


_TP = C.POINTER(OrcTensor)


class OrcModel(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("d_model", C.c_int), ("d_head", C.c_int), ("d_ffn", C.c_int),
                ("vocab_size", C.c_int), ("rope_freq_base", C.c_float),
                ("rms_norm_eps", C.c_float), ("no_rope_layer_interval", C.c_int),
                ("matmul_lanes", C.c_int),
                ("token_embd", OrcTensor), ("output_norm", OrcTensor), ("output", OrcTensor),
                ("attn_norm", _TP), ("attn_q", _TP), ("attn_k", _TP), ("attn_v", _TP),
                ("attn_output", _TP), ("attn_q_norm", _TP), ("attn_k_norm", _TP),
                ("ffn_norm", _TP), ("ffn_gate", _TP), ("ffn_up", _TP), ("ffn_down", _TP)]


def _load(path, what):
    if not os.path.exists(path):
        raise FileNotFoundError(f"{what} not built: {path} (run: make -C oracle {'ref' if 'ref' in what else ''})")
    return C.CDLL(path)


class Oracle:
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            L = _load(ORC_SO, "oracle")
            L.orc_f16_to_f32.restype = C.c_float
            L.orc_f16_to_f32.argtypes = [C.c_uint16]
            L.orc_dequant_row.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int]
            L.orc_matmul.argtypes = [_fp, C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
            L.orc_rms_norm.argtypes = [_fp, _fp, _fp, C.c_int, C.c_float]
            L.orc_softmax.argtypes = [_fp, C.c_int]
            L.orc_swiglu.argtypes = [_fp, _fp, _fp, C.c_int]
            L.orc_rope_apply.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
            L.orc_session_new.restype = C.c_void_p
            L.orc_session_new.argtypes = [C.POINTER(OrcModel), C.c_int]
            L.orc_session_free.argtypes = [C.c_void_p]
            L.orc_session_reset.argtypes = [C.c_void_p]
            L.orc_set_kv_f16.argtypes = [C.c_int]
            L.orc_set_kv_f16.restype = None
            L.orc_session_n_tokens.argtypes = [C.c_void_p]
            L.orc_forward.restype = _fp
            L.orc_forward.argtypes = [C.POINTER(OrcModel), C.c_void_p, C.c_int32, C.c_int]
            L.orc_rng_seed.argtypes = [_u64p, C.c_uint]
            L.orc_rng_next.restype = C.c_uint64
            L.orc_rng_next.argtypes = [_u64p]
            L.orc_apply_repeat_penalty.argtypes = [_fp, C.c_int, _ip, C.c_int, C.c_float]
            L.orc_sample.restype = C.c_int32
            L.orc_sample.argtypes = [_fp, C.c_int, C.POINTER(GenParams), _u64p]
            L.orc_generate_ids.argtypes = [C.POINTER(OrcModel), C.c_void_p, _ip, C.c_int,
                                           C.POINTER(GenParams), C.c_int32, _ip, C.c_int, _fp, C.c_int]
            cls._lib = L
        return cls._lib

    # -- block-level helpers ------------------------------------------------
    @classmethod
    def dequant(cls, blob: np.ndarray, n: int, dtype: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        cls.lib().orc_dequant_row(blob.ctypes.data, fptr(out), n, dtype)
        return out

    @classmethod
    def matmul(cls, a: np.ndarray, b: np.ndarray, m: int, k: int, n: int, dtype: int, lanes=16):
        out = np.zeros(m * n, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        cls.lib().orc_matmul(fptr(out), a.ctypes.data, fptr(b), m, k, n, dtype, lanes)
        return out.reshape(m, n)


class OracleModel:
    """The C restatement over a GGUF file (tensors stay in the mmap)."""

    def __init__(self, gguf, lanes: int = 16):
        from libcmol_b200.synth import GGUFFile
        self.g = gguf if isinstance(gguf, GGUFFile) else GGUFFile(gguf)
        hp = self.g.hparams()
        self.hp = hp
        self.L = Oracle.lib()
        m = OrcModel()
        for k in ("n_layers", "n_heads", "n_kv_heads", "d_model", "d_head", "d_ffn", "vocab_size"):
            setattr(m, k, hp[k])
        m.rope_freq_base = hp["rope_base"]
        m.rms_norm_eps = hp["rms_eps"]
        m.no_rope_layer_interval = hp["no_rope_interval"]
        m.matmul_lanes = lanes
        T = self.g.tensors

        def t(name):
            if name not in T:
                return OrcTensor(None, 0)
            dt, _, view = T[name]
            return OrcTensor(view.ctypes.data, dt)

        m.token_embd = t("token_embd.weight")
        m.output_norm = t("output_norm.weight")
        m.output = t("output.weight")
        self._arrays = []
        for fld, suf in (("attn_norm", "attn_norm"), ("attn_q", "attn_q"), ("attn_k", "attn_k"),
                         ("attn_v", "attn_v"), ("attn_output", "attn_output"),
                         ("attn_q_norm", "attn_q_norm"), ("attn_k_norm", "attn_k_norm"),
                         ("ffn_norm", "ffn_norm"), ("ffn_gate", "ffn_gate"), ("ffn_up", "ffn_up"),
                         ("ffn_down", "ffn_down")):
            arr = (OrcTensor * hp["n_layers"])(*[t(f"blk.{i}.{suf}.weight") for i in range(hp["n_layers"])])
            self._arrays.append(arr)
            setattr(m, fld, C.cast(arr, _TP))
        self.m = m

    def session(self, max_ctx: int):
        s = self.L.orc_session_new(C.byref(self.m), max_ctx)
        if not s:
            raise MemoryError("orc_session_new")
        return s

    def free_session(self, s):
        self.L.orc_session_free(s)

    def forward(self, s, tok: int, pos: int) -> np.ndarray:
        p = self.L.orc_forward(C.byref(self.m), s, tok, pos)
        if not p:
            raise RuntimeError("orc_forward failed")
        return np.ctypeslib.as_array(p, shape=(self.hp["vocab_size"],)).copy()

    def generate_ids(self, s, prompt, params: GenParams, eos=-1, out_cap=4096, logits_cap=0):
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(out_cap, np.int32)
        V = self.hp["vocab_size"]
        lg = np.zeros((max(logits_cap, 1), V), np.float32)
        n = self.L.orc_generate_ids(C.byref(self.m), s, iptr(prompt), len(prompt), C.byref(params),
                                    eos, iptr(out), out_cap, fptr(lg) if logits_cap else None, logits_cap)
        if n < 0:
            raise RuntimeError(f"orc_generate_ids: {n}")
        return out[:n], (lg[:min(n, logits_cap)] if logits_cap else None)


class Reference:
    """The unmodified reference library (oracle/_ref/libcmolref.so)."""
    _lib = None

    @classmethod
    def available(cls):
        return os.path.exists(REF_SO)

    @classmethod
    def lib(cls):
        if cls._lib is None:
            L = _load(REF_SO, "reference (make -C oracle ref)")
            L.cmol_load.restype = C.c_void_p
            L.cmol_load.argtypes = [C.c_char_p, C.c_void_p, C.POINTER(C.c_int)]
            L.cmol_free.argtypes = [C.c_void_p]
            L.cmol_session_acquire.restype = C.c_void_p
            L.cmol_session_acquire.argtypes = [C.c_void_p]
            L.cmol_session_release.argtypes = [C.c_void_p]
            L.cmol_session_reset.argtypes = [C.c_void_p]
            L.ref_kernel_name.restype = C.c_char_p
            L.ref_dequant_row.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int]
            L.ref_matmul.argtypes = [_fp, C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
            L.ref_rms_norm.argtypes = [_fp, _fp, _fp, C.c_int, C.c_float]
            L.ref_rope_apply.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
            L.ref_swiglu.argtypes = [_fp, _fp, _fp, C.c_int]
            L.ref_softmax.argtypes = [_fp, C.c_int]
            L.ref_rng_seed.argtypes = [_u64p, C.c_uint]
            L.ref_rng_next.restype = C.c_uint64
            L.ref_rng_next.argtypes = [_u64p]
            L.ref_repeat_penalty.argtypes = [_fp, C.c_int, _ip, C.c_int, C.c_float]
            L.ref_sample.restype = C.c_int32
            L.ref_sample.argtypes = [_fp, C.c_int, C.POINTER(GenParams), _u64p]
            L.ref_vocab_size.argtypes = [C.c_void_p]
            L.ref_eos_id.argtypes = [C.c_void_p]
            L.ref_n_tokens.argtypes = [C.c_void_p]
            L.ref_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int, _fp]
            L.ref_generate_ids.argtypes = [C.c_void_p, _ip, C.c_int, C.POINTER(GenParams), C.c_int32,
                                           _ip, C.c_int, _fp, C.c_int]
            L.cmol_encode.argtypes = [C.c_void_p, C.c_char_p, _ip, C.c_int]
            L.cmol_decode_token.restype = C.c_void_p
            L.cmol_decode_token.argtypes = [C.c_void_p, C.c_int32]
            L.cmol_strerror.restype = C.c_char_p
            L.cmol_strerror.argtypes = [C.c_int]
            L.cmol_format_chatml.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, C.c_size_t]
            L.cmol_format_chatml_turn.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
            cls._lib = L
        return cls._lib

    @classmethod
    def dequant(cls, blob, n, dtype):
        out = np.zeros(n, np.float32)
        cls.lib().ref_dequant_row(blob.ctypes.data, fptr(out), n, dtype)
        return out

    @classmethod
    def matmul(cls, a, b, m, k, n, dtype, which=1):
        out = np.zeros(m * n, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        cls.lib().ref_matmul(fptr(out), a.ctypes.data, fptr(b), m, k, n, dtype, which)
        return out.reshape(m, n)


class CmolConfig(C.Structure):
    _fields_ = [("max_ctx", C.c_int), ("max_sessions", C.c_int), ("prefill_chunk", C.c_int),
                ("log_fn", C.c_void_p), ("log_ud", C.c_void_p)]


class ReferenceModel:
    def __init__(self, path: str, max_ctx: int, max_sessions: int = 1):
        self.L = Reference.lib()
        cfg = CmolConfig(max_ctx, max_sessions, 512, None, None)
        err = C.c_int(0)
        self.m = self.L.cmol_load(path.encode(), C.byref(cfg), C.byref(err))
        if not self.m:
            raise RuntimeError(f"reference cmol_load failed: {err.value}")
        self.V = self.L.ref_vocab_size(self.m)

    def close(self):
        if self.m:
            self.L.cmol_free(self.m)
            self.m = None

    def session(self):
        """acquire + reset: the reference's acquire keeps the slot's old KV
        length (src/api.c:309-320), so a fresh session needs the reset."""
        s = self.L.cmol_session_acquire(self.m)
        if not s:
            raise RuntimeError("no session")
        self.L.cmol_session_reset(s)
        return s

    def release(self, s):
        self.L.cmol_session_release(s)

    def forward(self, s, tok, pos):
        out = np.zeros(self.V, np.float32)
        rc = self.L.ref_forward(self.m, s, tok, pos, fptr(out))
        if rc:
            raise RuntimeError("ref forward failed")
        return out

    def encode(self, text: str, cap: int = 4096):
        out = np.zeros(cap, np.int32)
        n = self.L.cmol_encode(self.m, text.encode(), iptr(out), cap)
        return n, out[:max(n, 0)]

    def decode_token(self, tid: int):
        p = self.L.cmol_decode_token(self.m, tid)
        return None if not p else C.string_at(p)

    def generate_ids(self, s, prompt, params: GenParams, eos=-1, out_cap=4096, logits_cap=0):
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(out_cap, np.int32)
        lg = np.zeros((max(logits_cap, 1), self.V), np.float32)
        n = self.L.ref_generate_ids(s, iptr(prompt), len(prompt), C.byref(params), eos, iptr(out),
                                    out_cap, fptr(lg) if logits_cap else None, logits_cap)
        if n < 0:
            raise RuntimeError(f"ref_generate_ids: {n}")
        return out[:n], (lg[:min(n, logits_cap)] if logits_cap else None)
