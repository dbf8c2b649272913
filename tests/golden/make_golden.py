"""Write the golden fixtures of tests/golden/ from the reference itself.

Run where the reference sources exist (builds oracle/_ref/libcmolref.so from
them with `make -C oracle ref`):

    python tests/golden/make_golden.py [gemv|models|configs|sampler|tokenizer ...]

(no argument: every section; the named sections only otherwise).

Every expected value below is produced by the UNMODIFIED reference
(nvlass/libcmol, compiled from its own src/cmol.c) through its exported
functions: cmol_dequant_row, the selected and the scalar matmul kernels,
cmol_model_forward (teacher forcing), the src/api.c generate loop with token
ids, cmol_sample / cmol_rng_seed / cmol_apply_repeat_penalty, and
cmol_encode / cmol_decode_token.  Q4_0 is not implemented by the
reference; its expected values come from gguf-py 0.19.0 `dequantize`.

The synthetic GGUF files are not stored: libcmol_b200.synth rebuilds them
deterministically from their spec; their SHA-256 is recorded so a test can
tell when the writer changed.
"""

from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from libcmol_b200 import synth  # noqa: E402

# Tiny model specs of the fixtures (vocab 512, 2-3 layers).
MODEL_SPECS = {
    "q8_0": dict(dtype=synth.Q8_0),
    "q5_0": dict(dtype=synth.Q5_0),
    "q4_k": dict(dtype=synth.Q4_K),
    "q6_k": dict(dtype=synth.Q6_K),
    # SmolLM3-style: NoPE every 2nd layer, rope base 5e6, QK-norm, untied head
    "smollm3": dict(dtype=synth.Q4_K, n_layers=3, arch="smollm3", no_rope_interval=2,
                    rope_base=5e6, qk_norm=True, tied=False, dt_head=synth.Q8_0, n_heads=4, n_kv_heads=1),
    # config-3 style mix: Q5_0 attention, Q4_K FFN, Q8_0 embedding, eos present
    "mixed": dict(dtype=synth.Q8_0, dt_attn=synth.Q5_0, dt_ffn=synth.Q4_K, dt_embd=synth.Q8_0, eos=2),
}


# Reduced-depth models that keep each BASELINE config's per-layer shape:
# d_model, heads / kv heads (G = 3, 3, 1, 4), d_head (64, 64, 64, 128),
# d_ffn, vocabulary (49152 or 128256), formats, RoPE base and NoPE rule.
# Config 4 keeps 4 layers so that its NoPE layer (every 4th) is present.
CONFIG_LAYERS = {1: 2, 2: 2, 3: 2, 4: 4}
CONFIG_TF_TOKENS = 24              # teacher-forced positions per config model
CONFIG_FULL_AT = (0, 23)           # positions whose full logit vectors are stored
CONFIG_TOPN = 32                   # top logits stored for every position


def config_spec(cfg):
    spec = synth.baseline_spec(cfg, ctx=512)
    spec.n_layers = CONFIG_LAYERS[cfg]
    spec.name = f"golden-config{cfg}-L{spec.n_layers}"
    return spec


def config_path(cfg, tmpdir):
    p = os.path.join(tmpdir, f"golden_config{cfg}.gguf")
    if not os.path.exists(p):
        synth.write_gguf(p, config_spec(cfg))
    return p


def model_spec(name):
    kw = dict(MODEL_SPECS[name])
    dt = kw.pop("dtype")
    spec = synth.tiny_spec(dt, **kw)
    spec.name = f"golden-{name}"
    return spec


def gguf_path(name, tmpdir):
    p = os.path.join(tmpdir, f"golden_{name}.gguf")
    synth.write_gguf(p, model_spec(name))
    return p


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 20), b""):
            h.update(b)
    return h.hexdigest()


def main():
    subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all", "ref"])
    from oracle.oracle import GenParams, Reference, ReferenceModel, fptr, iptr

    want = set(sys.argv[1:]) or {"gemv", "models", "configs", "sampler", "tokenizer"}
    R = Reference.lib()
    mpath = os.path.join(HERE, "manifest.json")
    manifest = json.load(open(mpath)) if os.path.exists(mpath) else {}
    manifest["kernel"] = R.ref_kernel_name().decode()
    manifest.setdefault("models", {})
    manifest.setdefault("configs", {})
    tmp = tempfile.mkdtemp(prefix="cmol_golden_")

    if "gemv" in want:
        # ---- GEMV / dequant on identical blocks -------------------------------
        gem = {}
        for dt in (synth.Q8_0, synth.Q5_0, synth.Q4_K, synth.Q6_K, synth.F16, synth.F32):
            name = synth.DTYPE_NAMES[dt]
            rng = np.random.default_rng(100 + dt)
            m, k = 12, 512
            blob = synth.quantize(rng.standard_normal((m, k), dtype=np.float32) * 0.02, dt)
            for n in (1, 3):
                x = rng.standard_normal((k, n), dtype=np.float32)
                gem[f"{name}_n{n}_blocks"] = blob
                gem[f"{name}_n{n}_x"] = x
                gem[f"{name}_n{n}_simd"] = Reference.matmul(blob, x, m, k, n, dt, which=1)
                gem[f"{name}_n{n}_scalar"] = Reference.matmul(blob, x, m, k, n, dt, which=0)
            gem[f"{name}_deq_row0"] = Reference.dequant(blob[0], k, dt)
        # Q4_0: gguf-py (the reference has no Q4_0)
        from gguf import GGMLQuantizationType, quants
        rng = np.random.default_rng(7)
        q40 = synth.quantize(rng.standard_normal((4, 256), dtype=np.float32) * 0.02, synth.Q4_0)
        gem["Q4_0_blocks"] = q40
        gem["Q4_0_deq_ggufpy"] = quants.dequantize(q40, GGMLQuantizationType.Q4_0).astype(np.float32)
        np.savez_compressed(os.path.join(HERE, "gemv.npz"), **gem)

    if "models" in want:
        # ---- models: teacher-forced logits + generate loops --------------------
        toks = [5, 300, 17, 99, 400, 12, 260, 261, 77, 1, 2, 3, 450, 33]
        mod = {}
        for name in MODEL_SPECS:
            path = gguf_path(name, tmp)
            manifest["models"][name] = {"sha256": sha256(path), "spec": MODEL_SPECS[name] | {"dtype": None}}
            rm = ReferenceModel(path, 64)
            s = rm.session()
            mod[f"{name}_tokens"] = np.array(toks, np.int32)
            mod[f"{name}_logits"] = np.stack([rm.forward(s, t, i) for i, t in enumerate(toks)])
            rm.release(s)
            eos = rm.L.ref_eos_id(rm.m)
            for tag, p in (("greedy", GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20)),
                           ("greedy_pen", GenParams.make(0.0, repeat_penalty=1.3, repeat_last_n=8, max_new_tokens=20)),
                           ("topp", GenParams.make(0.9, top_p=0.9, top_k=40, seed=1234, repeat_penalty=1.1,
                                                   max_new_tokens=20)),
                           ("topk", GenParams.make(1.2, top_p=1.0, top_k=5, seed=99, repeat_penalty=1.0,
                                                   max_new_tokens=20))):
                s = rm.session()
                ids, lg = rm.generate_ids(s, toks[:6], p, eos=eos, logits_cap=32)
                mod[f"{name}_gen_{tag}"] = ids
                mod[f"{name}_gen_{tag}_logits"] = lg
                rm.release(s)
            rm.close()
        np.savez_compressed(os.path.join(HERE, "models.npz"), **mod)

    if "configs" in want:
        # ---- config shapes: teacher-forced logits and streams ------------------
        # Configs 1, 3 and 4 from the reference; config 2 is Q4_0, which the
        # reference does not implement (src/quant.c:298-308), so its values come
        # from the C restatement (oracle/cmol_oracle.c), whose Q4_0 block decode
        # is pinned to gguf-py's dequantize and whose every other step is pinned
        # to the reference by the fixtures above.
        from oracle.oracle import OracleModel
        cfgs = {}
        for cfg in (1, 2, 3, 4):
            path = config_path(cfg, tmp)
            spec = config_spec(cfg)
            manifest["configs"][str(cfg)] = {"sha256": sha256(path), "name": spec.name, "n_layers": spec.n_layers,
                                             "source": "oracle (Q4_0)" if cfg == 2 else "reference"}
            rng = np.random.default_rng(500 + cfg)
            V = spec.vocab_size
            toks = rng.integers(0, V, size=CONFIG_TF_TOKENS).astype(np.int32)
            params = {"greedy": GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=12),
                      "topp": GenParams.make(0.9, top_p=0.9, top_k=40, seed=77, repeat_penalty=1.1,
                                             max_new_tokens=12)}
            if cfg == 2:
                om = OracleModel(path, lanes=16)
                s_ = om.session(64)
                lg = np.stack([om.forward(s_, int(t), i) for i, t in enumerate(toks)])
                om.free_session(s_)
                gens = {}
                for tag, p in params.items():
                    s_ = om.session(64)
                    ids, _ = om.generate_ids(s_, toks[:6], p)
                    gens[tag] = ids
                    om.free_session(s_)
            else:
                rm = ReferenceModel(path, 64)
                s_ = rm.session()
                lg = np.stack([rm.forward(s_, int(t), i) for i, t in enumerate(toks)])
                rm.release(s_)
                gens = {}
                for tag, p in params.items():
                    s_ = rm.session()
                    ids, _ = rm.generate_ids(s_, toks[:6], p)
                    gens[tag] = ids
                    rm.release(s_)
                rm.close()
            top = np.argsort(-lg, axis=1, kind="stable")[:, :CONFIG_TOPN].astype(np.int32)
            cfgs[f"c{cfg}_tokens"] = toks
            cfgs[f"c{cfg}_top_ids"] = top
            cfgs[f"c{cfg}_top_vals"] = np.take_along_axis(lg, top, axis=1)
            cfgs[f"c{cfg}_norm"] = np.linalg.norm(lg, axis=1).astype(np.float32)
            for at in CONFIG_FULL_AT:
                cfgs[f"c{cfg}_full{at}"] = lg[at]
            for tag, ids in gens.items():
                cfgs[f"c{cfg}_gen_{tag}"] = np.asarray(ids, np.int32)
            os.remove(path)
        np.savez_compressed(os.path.join(HERE, "configs.npz"), **cfgs)

    if "sampler" in want:
        # ---- sampler on identical logits --------------------------------------
        smp = {"logits": [], "params": [], "ring": [], "token": [], "rng_after": []}
        rng = np.random.default_rng(11)
        for case in range(48):
            V = 1000
            lg = (rng.standard_normal(V) * (0.5 + case % 4)).astype(np.float32)
            if case % 6 == 5:
                lg[rng.integers(V, size=20)] = lg.max()          # exact ties at the top
            temp = [0.0, 0.7, 1.0, 1.5][case % 4]
            top_k = [0, 1, 40, 600][(case // 4) % 4]
            top_p = [1.0, 0.9, 0.5][(case // 16) % 3]
            pen = [1.0, 1.1, 2.0][case % 3]
            seed = 1000 + case
            ring = rng.integers(V, size=int(rng.integers(0, 40))).astype(np.int32)
            p = GenParams.make(temp, top_p=top_p, top_k=top_k, seed=seed, repeat_penalty=pen)
            st = (np.ctypeslib.ctypes.c_uint64 * 4)()
            R.ref_rng_seed(st, seed)
            work = lg.copy()
            if pen > 1.0 and len(ring):
                R.ref_repeat_penalty(fptr(work), V, iptr(ring), len(ring), pen)
            tok = R.ref_sample(fptr(work), V, p, st)
            smp["logits"].append(lg)
            smp["params"].append([temp, top_p, top_k, pen, seed])
            smp["ring"].append(np.pad(ring, (0, 64 - len(ring)), constant_values=-1))
            smp["token"].append(tok)
            smp["rng_after"].append(np.array(list(st), np.uint64))
        np.savez_compressed(os.path.join(HERE, "sampler.npz"),
                            **{k: np.array(v) for k, v in smp.items()})

    if "tokenizer" in want:
        # ---- tokenizer ---------------------------------------------------------
        texts = ["hello world", "  two  spaces", "<|im_start|>user\nhi<|im_end|>", "abc xyz q",
                 "café ☃ snow", "", "a" * 300, "tab\there", "x<|im_end|>y<|endoftext|>"]
        path = gguf_path("q8_0", tmp)
        rm = ReferenceModel(path, 64)
        tk = {"texts": texts, "encode": [], "decode": {}}
        for t in texts:
            n, ids = rm.encode(t)
            tk["encode"].append({"rc": int(n), "ids": [int(i) for i in ids]})
        for tid in list(range(0, 300, 7)) + [358, 359, 400, 511]:
            b = rm.decode_token(tid)
            tk["decode"][str(tid)] = None if b is None else b.hex()
        tk["strerror"] = {str(c): R.cmol_strerror(c).decode() for c in range(-9, 1)}
        rm.close()
        with open(os.path.join(HERE, "tokenizer.json"), "w") as f:
            json.dump(tk, f, indent=1)

    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    import shutil
    shutil.rmtree(tmp, ignore_errors=True)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
