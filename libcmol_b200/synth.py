"""Seeded synthetic GGUF models for the libcmol decode path.

There is no network and no real checkpoint here, so every model this package
tests or benchmarks is written by this module: a SmolLM2/SmolLM3-shaped
decoder with N(0, 0.02) weights, RMSNorm gains 1.0, block-quantised into the
GGUF formats the reference reads (block layouts of src/quant.c:78-105 of the
reference; Q4_0 from the GGUF/ggml format).  The file carries every metadata
key the reference loader needs (src/gguf.c:57-79, including
``{arch}.vocab_size`` which cmol_gguf_peek requires, src/gguf.c:604), F32
norm weights (read as raw float*, src/model.c:225) and a synthetic
SentencePiece-style BPE vocabulary with byte-fallback tokens and merges.

Any valid block encoding works for parity, because the engine and the
checkers are always compared on the identical blocks read from the file.
"""

from __future__ import annotations

import dataclasses
import mmap
import os
import struct

import numpy as np

# GGUF tensor type tags (src/cmol_internal.h:27-37 of the reference)
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 6, 8, 12, 14
DTYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q5_0: "Q5_0",
               Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q5_0: (32, 22),
         Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def row_bytes(k: int, dtype: int) -> int:
    bv, bb = BLOCK[dtype]
    return (k // bv) * bb


# ---------------------------------------------------------------------------
# Block quantisers (numpy, vectorised over rows).  Input: float32 [M, K].
# Output: uint8 [M, row_bytes].
# ---------------------------------------------------------------------------

def _f16(x):
    return x.astype(np.float16)


def _signed_absmax(b):
    idx = np.abs(b).argmax(axis=-1)
    return np.take_along_axis(b, idx[..., None], axis=-1)[..., 0]


def quantize_q8_0(w):
    M, K = w.shape
    b = w.reshape(M, K // 32, 32)
    d16 = _f16(np.abs(b).max(-1) / 127.0)
    d = d16.astype(np.float32)
    inv = np.divide(1.0, d, out=np.zeros_like(d), where=d > 0)
    q = np.clip(np.rint(b * inv[..., None]), -127, 127).astype(np.int8)
    out = np.empty((M, K // 32, 34), np.uint8)
    out[..., 0:2] = d16.view(np.uint8).reshape(M, K // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(M, -1)


def quantize_q4_0(w):
    M, K = w.shape
    b = w.reshape(M, K // 32, 32)
    d16 = _f16(_signed_absmax(b) / -8.0)
    d = d16.astype(np.float32)
    inv = np.divide(1.0, d, out=np.zeros_like(d), where=d != 0)
    q = np.clip(np.floor(b * inv[..., None] + 8.5), 0, 15).astype(np.uint8)
    out = np.empty((M, K // 32, 18), np.uint8)
    out[..., 0:2] = d16.view(np.uint8).reshape(M, K // 32, 2)
    out[..., 2:] = q[..., :16] | (q[..., 16:] << 4)
    return out.reshape(M, -1)


def quantize_q5_0(w):
    M, K = w.shape
    b = w.reshape(M, K // 32, 32)
    d16 = _f16(_signed_absmax(b) / -16.0)
    d = d16.astype(np.float32)
    inv = np.divide(1.0, d, out=np.zeros_like(d), where=d != 0)
    q = np.clip(np.floor(b * inv[..., None] + 16.5), 0, 31).astype(np.uint32)
    qh = (((q >> 4) & 1) << np.arange(32, dtype=np.uint32)).sum(-1).astype(np.uint32)
    out = np.empty((M, K // 32, 22), np.uint8)
    out[..., 0:2] = d16.view(np.uint8).reshape(M, K // 32, 2)
    out[..., 2:6] = qh.view(np.uint8).reshape(M, K // 32, 4)
    out[..., 6:] = ((q[..., :16] & 15) | ((q[..., 16:] & 15) << 4)).astype(np.uint8)
    return out.reshape(M, -1)


def quantize_q4_k(w):
    M, K = w.shape
    nb = K // 256
    b = w.reshape(M, nb, 8, 32)
    mn = np.minimum(b.min(-1), 0.0)
    mx = b.max(-1)
    scale = (mx - mn) / 15.0
    minv = -mn
    d16 = _f16(scale.max(-1) / 63.0)
    dm16 = _f16(minv.max(-1) / 63.0)
    d = d16.astype(np.float32)[..., None]
    dm = dm16.astype(np.float32)[..., None]
    sc = np.clip(np.rint(np.divide(scale, d, out=np.zeros_like(scale), where=d > 0)), 0, 63).astype(np.uint8)
    mi = np.clip(np.rint(np.divide(minv, dm, out=np.zeros_like(minv), where=dm > 0)), 0, 63).astype(np.uint8)
    dl = (d * sc.astype(np.float32))[..., None]
    ml = (dm * mi.astype(np.float32))[..., None]
    q = np.clip(np.rint(np.divide(b + ml, dl, out=np.zeros_like(b), where=dl > 0)), 0, 15).astype(np.uint8)
    s12 = np.zeros((M, nb, 12), np.uint8)
    s12[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    s12[..., 4:8] = mi[..., 0:4] | ((mi[..., 4:8] >> 4) << 6)
    s12[..., 8:12] = (sc[..., 4:8] & 15) | ((mi[..., 4:8] & 15) << 4)
    qs = (q[:, :, 0::2, :] | (q[:, :, 1::2, :] << 4)).reshape(M, nb, 128)
    out = np.empty((M, nb, 144), np.uint8)
    out[..., 0:2] = d16.view(np.uint8).reshape(M, nb, 2)
    out[..., 2:4] = dm16.view(np.uint8).reshape(M, nb, 2)
    out[..., 4:16] = s12
    out[..., 16:] = qs
    return out.reshape(M, -1)


def quantize_q6_k(w):
    M, K = w.shape
    nb = K // 256
    b = w.reshape(M, nb, 16, 16)
    scale = _signed_absmax(b) / -32.0
    amax = np.abs(scale).max(-1)
    d16 = _f16(amax / 127.0)
    d = d16.astype(np.float32)[..., None]
    sc = np.clip(np.rint(np.divide(scale, d, out=np.zeros_like(scale), where=d > 0)), -128, 127).astype(np.int8)
    dl = (d * sc.astype(np.float32))[..., None]
    q = np.clip(np.rint(np.divide(b, dl, out=np.zeros_like(b), where=dl != 0)) + 32, 0, 63).astype(np.uint8)
    q = q.reshape(M, nb, 256)
    lo, hi = q & 15, q >> 4
    ql = np.zeros((M, nb, 128), np.uint8)
    qh = np.zeros((M, nb, 64), np.uint8)
    j = np.arange(32)
    for g in range(8):
        li = (0 if g < 4 else 64) + (g & 1) * 32 + j
        ql[..., li] |= lo[..., g * 32:(g + 1) * 32] << (4 if g & 2 else 0)
        hj = (0 if g < 4 else 32) + j
        qh[..., hj] |= hi[..., g * 32:(g + 1) * 32] << ((g & 3) * 2)
    out = np.empty((M, nb, 210), np.uint8)
    out[..., 0:128] = ql
    out[..., 128:192] = qh
    out[..., 192:208] = sc.view(np.uint8)
    out[..., 208:210] = d16.view(np.uint8).reshape(M, nb, 2)
    return out.reshape(M, -1)


def quantize(w, dtype):
    w = np.ascontiguousarray(w, dtype=np.float32)
    if dtype == F32:
        return w.view(np.uint8).reshape(w.shape[0], -1)
    if dtype == F16:
        return w.astype(np.float16).view(np.uint8).reshape(w.shape[0], -1)
    return {Q8_0: quantize_q8_0, Q4_0: quantize_q4_0, Q5_0: quantize_q5_0,
            Q4_K: quantize_q4_k, Q6_K: quantize_q6_k}[dtype](w)


# ---------------------------------------------------------------------------
# Model shapes
# ---------------------------------------------------------------------------

@dataclasses.dataclass
class ModelSpec:
    name: str
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    d_ffn: int
    vocab_size: int
    ctx: int = 2048
    rope_base: float = 10000.0
    rms_eps: float = 1e-5
    arch: str = "llama"
    no_rope_interval: int = 0
    tied: bool = True
    qk_norm: bool = False
    dt_attn: int = Q8_0
    dt_ffn: int = Q8_0
    dt_embd: int = Q8_0
    dt_head: int = Q8_0          # only used when not tied
    eos: int = -1                # -1: no eos key (generation never stops on EOS)
    seed: int = 1234

    @property
    def d_head(self):
        return self.d_model // self.n_heads

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.d_head


def baseline_spec(cfg: int, ctx: int | None = None) -> ModelSpec:
    """The five model shapes of the benchmark configs (1-based)."""
    if cfg == 1:
        s = ModelSpec("smollm2-135m-q8_0", 30, 576, 9, 3, 1536, 49152, ctx=2048)
    elif cfg == 2:
        s = ModelSpec("smollm2-360m-q4_0", 32, 960, 15, 5, 2560, 49152, ctx=2048,
                      dt_attn=Q4_0, dt_ffn=Q4_0, dt_embd=Q4_0)
    elif cfg == 3:
        s = ModelSpec("smollm2-1.7b-q5_0-q4_k", 24, 2048, 32, 32, 8192, 49152, ctx=2048,
                      dt_attn=Q5_0, dt_ffn=Q4_K, dt_embd=Q8_0)
    elif cfg == 4:
        s = ModelSpec("smollm3-3b-q4_k", 36, 2048, 16, 4, 11008, 128256, ctx=8192 + 512,
                      rope_base=5e6, arch="smollm3", no_rope_interval=4, tied=False,
                      dt_attn=Q4_K, dt_ffn=Q4_K, dt_embd=Q4_K, dt_head=Q8_0)
    else:
        raise ValueError(cfg)
    if ctx:
        s.ctx = ctx
    return s


def tiny_spec(dtype=Q8_0, **kw) -> ModelSpec:
    """A small model for parity tests (runs through the CPU checkers in ms)."""
    base = dict(name="tiny", n_layers=2, d_model=256, n_heads=4, n_kv_heads=2,
                d_ffn=512, vocab_size=512, ctx=128, dt_attn=dtype, dt_ffn=dtype,
                dt_embd=dtype if BLOCK[dtype][0] <= 256 else Q8_0)
    base.update(kw)
    return ModelSpec(**base)


# ---------------------------------------------------------------------------
# Synthetic BPE vocabulary
# ---------------------------------------------------------------------------

SP = "▁"
CONTROL, NORMAL, BYTE = 3, 1, 6


def synth_vocab(V: int, seed: int = 7):
    """tokens, scores, types, merges for a SentencePiece-style vocabulary."""
    toks = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]
    types = [CONTROL] * 3
    toks += ["<0x%02X>" % i for i in range(256)]
    types += [BYTE] * 256
    base = [SP] + [chr(c) for c in range(0x21, 0x7F)]
    toks += base
    types += [NORMAL] * len(base)
    if V < len(toks):
        raise ValueError("vocab too small")
    rng = np.random.default_rng(seed)
    seen = set(toks)
    merges = []
    normal = list(base)
    letters = [chr(c) for c in range(0x61, 0x7B)]
    # seed merges: "▁"+letter and letter pairs make realistic words
    cands = [(SP, a) for a in letters] + [(a, b) for a in letters for b in letters]
    ci = 0
    while len(toks) < V:
        if ci < len(cands):
            a, b = cands[ci]
            ci += 1
        else:
            a = normal[int(rng.integers(len(normal)))]
            b = normal[int(rng.integers(min(len(normal), 200)))]
        s = a + b
        if s in seen or len(s.encode()) > 24:
            continue
        seen.add(s)
        toks.append(s)
        types.append(NORMAL)
        normal.append(s)
        merges.append(a + " " + b)
    scores = -np.arange(V, dtype=np.float32)
    return toks, scores, types, merges


# ---------------------------------------------------------------------------
# GGUF writer / reader (format: magic, version 3, counts, KV pairs, tensor
# infos, 32-byte aligned data — the layout src/gguf.c:448-518 parses)
# ---------------------------------------------------------------------------

GV_UINT32, GV_INT32, GV_FLOAT32, GV_BOOL, GV_STRING, GV_ARRAY = 4, 5, 6, 7, 8, 9
ALIGN = 32


def _s(x: str) -> bytes:
    b = x.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _kv(key, gtype, val):
    out = _s(key) + struct.pack("<I", gtype)
    if gtype == GV_UINT32:
        out += struct.pack("<I", val)
    elif gtype == GV_INT32:
        out += struct.pack("<i", val)
    elif gtype == GV_FLOAT32:
        out += struct.pack("<f", val)
    elif gtype == GV_BOOL:
        out += struct.pack("<B", 1 if val else 0)
    elif gtype == GV_STRING:
        out += _s(val)
    elif gtype == GV_ARRAY:
        et, items = val
        out += struct.pack("<IQ", et, len(items))
        if et == GV_STRING:
            out += b"".join(_s(x) for x in items)
        elif et == GV_FLOAT32:
            out += np.asarray(items, np.float32).tobytes()
        elif et == GV_INT32:
            out += np.asarray(items, np.int32).tobytes()
        else:
            raise ValueError(et)
    return out


def _tensor_plan(spec: ModelSpec):
    """(name, dtype, shape=(rows, k)) in file order."""
    D, F, KV, V = spec.d_model, spec.d_ffn, spec.kv_dim, spec.vocab_size
    plan = [("token_embd.weight", spec.dt_embd, (V, D))]
    for L in range(spec.n_layers):
        p = f"blk.{L}."
        plan += [(p + "attn_norm.weight", F32, (1, D)),
                 (p + "attn_q.weight", spec.dt_attn, (D, D)),
                 (p + "attn_k.weight", spec.dt_attn, (KV, D)),
                 (p + "attn_v.weight", spec.dt_attn, (KV, D)),
                 (p + "attn_output.weight", spec.dt_attn, (D, D))]
        if spec.qk_norm:
            plan += [(p + "attn_q_norm.weight", F32, (1, spec.d_head)),
                     (p + "attn_k_norm.weight", F32, (1, spec.d_head))]
        plan += [(p + "ffn_norm.weight", F32, (1, D)),
                 (p + "ffn_gate.weight", spec.dt_ffn, (F, D)),
                 (p + "ffn_up.weight", spec.dt_ffn, (F, D)),
                 (p + "ffn_down.weight", spec.dt_ffn, (D, F))]
    plan.append(("output_norm.weight", F32, (1, D)))
    if not spec.tied:
        plan.append(("output.weight", spec.dt_head, (V, D)))
    return plan


def _gen_tensor(spec, idx, name, dtype, shape, chunk_rows):
    rows, k = shape
    if name.endswith("norm.weight"):
        if "q_norm" in name or "k_norm" in name:
            g = np.random.default_rng([spec.seed, idx])
            yield (1.0 + 0.1 * g.standard_normal((1, k), dtype=np.float32)).astype(np.float32).view(np.uint8).reshape(1, -1)
            return
        yield np.ones((1, k), np.float32).view(np.uint8).reshape(1, -1)
        return
    g = np.random.default_rng([spec.seed, idx])
    for r0 in range(0, rows, chunk_rows):
        n = min(chunk_rows, rows - r0)
        w = g.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
        yield quantize(w, dtype)


def write_gguf(path: str, spec: ModelSpec, chunk_rows: int = 4096, workers: int | None = None):
    """Write the synthetic model; returns path.  Deterministic in spec.seed."""
    arch = spec.arch
    toks, scores, types, merges = synth_vocab(spec.vocab_size)
    kvs = [
        _kv("general.architecture", GV_STRING, arch),
        _kv("general.name", GV_STRING, spec.name),
        _kv(f"{arch}.context_length", GV_UINT32, spec.ctx),
        _kv(f"{arch}.embedding_length", GV_UINT32, spec.d_model),
        _kv(f"{arch}.block_count", GV_UINT32, spec.n_layers),
        _kv(f"{arch}.feed_forward_length", GV_UINT32, spec.d_ffn),
        _kv(f"{arch}.attention.head_count", GV_UINT32, spec.n_heads),
        _kv(f"{arch}.attention.head_count_kv", GV_UINT32, spec.n_kv_heads),
        _kv(f"{arch}.rope.freq_base", GV_FLOAT32, spec.rope_base),
        _kv(f"{arch}.attention.layer_norm_rms_epsilon", GV_FLOAT32, spec.rms_eps),
        _kv(f"{arch}.vocab_size", GV_UINT32, spec.vocab_size),
        _kv("tokenizer.ggml.model", GV_STRING, "llama"),
        _kv("tokenizer.ggml.tokens", GV_ARRAY, (GV_STRING, toks)),
        _kv("tokenizer.ggml.scores", GV_ARRAY, (GV_FLOAT32, scores)),
        _kv("tokenizer.ggml.token_type", GV_ARRAY, (GV_INT32, types)),
        _kv("tokenizer.ggml.merges", GV_ARRAY, (GV_STRING, merges)),
        _kv("tokenizer.ggml.bos_token_id", GV_UINT32, 1),
        _kv("tokenizer.ggml.add_bos_token", GV_BOOL, False),
    ]
    if spec.no_rope_interval:
        kvs.append(_kv(f"{arch}.attention.no_rope_layer_interval", GV_UINT32, spec.no_rope_interval))
    if spec.eos >= 0:
        kvs.append(_kv("tokenizer.ggml.eos_token_id", GV_UINT32, spec.eos))
    plan = _tensor_plan(spec)
    infos, off = [], 0
    for name, dt, (rows, k) in plan:
        nbytes = rows * row_bytes(k, dt)
        dims = (k,) if rows == 1 and name.endswith("norm.weight") else (k, rows)
        infos.append(_s(name) + struct.pack("<I", len(dims)) +
                     b"".join(struct.pack("<Q", x) for x in dims) +
                     struct.pack("<IQ", dt, off))
        off += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    head = b"GGUF" + struct.pack("<IQQ", 3, len(plan), len(kvs)) + b"".join(kvs) + b"".join(infos)
    pad = (-len(head)) % ALIGN
    tmp = path + ".tmp"
    data0 = len(head) + pad
    with open(tmp, "wb") as f:
        f.write(head + b"\0" * pad)
        f.truncate(data0 + off)
    offs, o = [], 0
    for name, dt, (rows, k) in plan:
        offs.append(o)
        o += (rows * row_bytes(k, dt) + ALIGN - 1) // ALIGN * ALIGN
    jobs = [(tmp, data0 + offs[i], spec, i, name, dt, shape, chunk_rows) for i, (name, dt, shape) in enumerate(plan)]
    if workers is None:
        workers = min(16, os.cpu_count() or 1) if off > (256 << 20) else 1
    done = False
    if workers > 1:
        # tensors are independent and seeded by index: fill them in parallel
        # (fresh "spawn" workers, never a fork of a process that may hold a GPU
        # context).  A pool that cannot start (e.g. a main module read from
        # stdin cannot be re-imported by spawn) raises; fall back to serial.
        import concurrent.futures as cf
        import multiprocessing as mp
        try:
            with cf.ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn")) as ex:
                for f in [ex.submit(_write_tensor, *j) for j in jobs]:
                    f.result(timeout=3600)
            done = True
        except Exception:
            done = False
    if not done:
        for j in jobs:
            _write_tensor(*j)
    os.replace(tmp, path)
    return path


def _write_tensor(tmp, at, spec, idx, name, dt, shape, chunk_rows):
    with open(tmp, "r+b") as f:
        f.seek(at)
        for blk in _gen_tensor(spec, idx, name, dt, shape, chunk_rows):
            f.write(blk.tobytes())


def ensure_gguf(path: str, spec: ModelSpec):
    if not os.path.exists(path):
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        write_gguf(path, spec)
    return path


class GGUFFile:
    """Minimal reader: metadata dict and tensors as uint8 views into an mmap."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self.mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.buf = np.frombuffer(self.mm, dtype=np.uint8)
        self.kv = {}
        self.tensors = {}
        self._parse()

    def close(self):
        self.buf = None
        self.tensors = {}
        try:
            self.mm.close()
        except BufferError:
            pass
        self._f.close()

    def _parse(self):
        mm = self.mm
        pos = 0

        def rd(fmt):
            nonlocal pos
            v = struct.unpack_from(fmt, mm, pos)
            pos += struct.calcsize(fmt)
            return v[0] if len(v) == 1 else v

        def rs():
            n = rd("<Q")
            nonlocal pos
            s = bytes(mm[pos:pos + n]).decode("utf-8", "replace")
            pos += n
            return s

        scal = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B",
                10: "<Q", 11: "<q", 12: "<d"}

        def rv(t):
            if t == GV_STRING:
                return rs()
            if t == GV_ARRAY:
                et, n = rd("<I"), rd("<Q")
                return [rv(et) for _ in range(n)]
            return rd(scal[t])

        magic = bytes(mm[0:4])
        if magic != b"GGUF":
            raise ValueError("not a GGUF file")
        pos = 4
        self.version = rd("<I")
        nt, nkv = rd("<Q"), rd("<Q")
        for _ in range(nkv):
            k = rs()
            t = rd("<I")
            self.kv[k] = rv(t)
        infos = []
        for _ in range(nt):
            name = rs()
            nd = rd("<I")
            dims = [rd("<Q") for _ in range(nd)]
            dt, off = rd("<I"), rd("<Q")
            infos.append((name, dims, dt, off))
        base = (pos + ALIGN - 1) // ALIGN * ALIGN
        for name, dims, dt, off in infos:
            k = dims[0]
            rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
            nbytes = rows * row_bytes(k, dt)
            self.tensors[name] = (dt, (rows, k), self.buf[base + off: base + off + nbytes])

    def arch(self):
        return self.kv.get("general.architecture", "llama")

    def hparams(self):
        a = self.arch()
        g = lambda s, d=0: self.kv.get(f"{a}.{s}", d)
        D, H = g("embedding_length"), g("attention.head_count")
        return dict(n_layers=g("block_count"), d_model=D, n_heads=H,
                    n_kv_heads=g("attention.head_count_kv", H) or H,
                    d_head=D // H if H else 0, d_ffn=g("feed_forward_length"),
                    vocab_size=g("vocab_size") or len(self.kv.get("tokenizer.ggml.tokens", [])),
                    ctx=g("context_length"), rope_base=float(g("rope.freq_base", 10000.0)),
                    rms_eps=float(g("attention.layer_norm_rms_epsilon", 1e-5)),
                    no_rope_interval=g("attention.no_rope_layer_interval", 0),
                    eos=self.kv.get("tokenizer.ggml.eos_token_id", -1))
