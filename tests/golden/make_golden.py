"""Regenerate the committed golden fixtures from the reference's OWN code.

Needs oracle/_ref/libvla_ref.so (oracle/Makefile builds it from the reference
checkout). Run from the repo root:  python tests/golden/make_golden.py

* act_<cfg>_m<mask>.npy  - actions [chunk, action_dim] of the reference's
  vla_act_predict (ACT_INT8=<mask>) on synth.write_act_checkpoint(seed=0) with
  synth.act_inputs(seed=1); cfg small = synth.ACT_SMALL, base = ACT_BASELINE.
* dp_<cfg>_m<mask>[_<variant>].npy - actions [chunk, action_dim] of the
  reference's vla_diffusion_predict (DIFFUSION_INT8=<mask>) on
  synth.write_dp_checkpoint(seed=0) with synth.dp_inputs(seed=1); variant
  ddpm = DP_SCHEDULER=DDPM (DP_STEPS=10), nonoise = a NULL noise pointer. The
  reference runs with OMP_NUM_THREADS=1: its GroupNorm splits the pixel sums
  per thread when a map has fewer than 16 channels per thread, so one thread
  is the order-defined result.
* checkpoints.json       - sha256 of each synthetic checkpoint directory, so a
  test notices if the writer ever stops reproducing the bytes the fixtures
  were made from.
* gemm.npz / gemm.json   - W8A8 linear cases (default_rng inputs): for small
  shapes the full xq / ascale / int32 accumulators / fp32 outputs, for the
  rest their sha256, all from the reference's quantize_act_i8,
  pack_weights_i8 and dense_linear_i8_ref.
"""
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

from oracle import oracle  # noqa: E402
from vla_simd_b200 import synth  # noqa: E402

ACT_CASES = [("small", synth.ACT_SMALL, 63), ("small", synth.ACT_SMALL, 0), ("small", synth.ACT_SMALL, 31),
             ("small", synth.ACT_SMALL, 40), ("base", synth.ACT_BASELINE, 63)]
# (seq_q, seq_k, n_q, n_kv): ACT encoder self, decoder self, decoder cross, GQA
ATTN_CASES = [(602, 602, 8, 8), (100, 100, 8, 8), (100, 602, 8, 8), (50, 113, 15, 5), (3, 40, 4, 2)]
LN_CASES = [(602, 512), (100, 512), (7, 960)]
F32_LINEAR_CASES = [(1, 512, 6), (100, 6, 512), (5, 10, 37), (640, 1024, 260), (37, 2048, 259)]   # (seq, N, K): state_proj, head, odd, DP cond (many rows)
# (cfg, shape name, DIFFUSION_INT8, variant)
DP_CASES = [("small", "DP_SMALL", 3, ""), ("small", "DP_SMALL", 0, ""), ("small", "DP_SMALL", 1, ""),
            ("small", "DP_SMALL", 3, "ddpm"), ("small", "DP_SMALL", 3, "nonoise"), ("base", "DP_BASELINE", 3, ""),
            ("base", "DP_BASELINE", 0, ""), ("edge", "DP_EDGE", 3, ""), ("edge", "DP_EDGE", 0, ""),
            ("edge", "DP_EDGE", 2, ""), ("deep", "DP_DEEP", 3, ""), ("deep", "DP_DEEP", 0, "")]
GEMM_SHAPES = [(1, 16, 3), (7, 48, 64), (13, 64, 17), (257, 96, 48), (50, 768, 1027), (602, 3200, 512),
               (602, 512, 3200), (300, 512, 512)]


def dir_digest(d):
    h = hashlib.sha256()
    for name in sorted(os.listdir(d)):
        if not os.path.isfile(os.path.join(d, name)):
            continue
        h.update(name.encode())
        with open(os.path.join(d, name), "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def gemm_inputs(seq, N, K, seed=11):
    rng = np.random.default_rng(seed + seq * 7 + N * 13 + K)
    x = rng.standard_normal((seq, K), dtype=np.float32)
    W = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    return x, W, b


def attn_inputs(sq, sk, nq, nkv, seed=21):
    rng = np.random.default_rng(seed + sq + 3 * sk + 7 * nq)
    Q = rng.standard_normal((sq, nq * 64), dtype=np.float32)
    K = rng.standard_normal((sk, nkv * 64), dtype=np.float32)
    V = rng.standard_normal((sk, nkv * 64), dtype=np.float32)
    return Q, K, V


def causal_mask(sq, sk):
    i = np.arange(sq)[:, None]
    j = np.arange(sk)[None, :]
    return np.where(j > i + (sk - sq), -np.inf, 0.0).astype(np.float32)


def ln_inputs(seq, H, seed=31):
    rng = np.random.default_rng(seed + seq + H)
    x = (rng.standard_normal((seq, H), dtype=np.float32) * np.float32(2.0) + np.float32(0.5)).astype(np.float32)
    w = (1.0 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    b = (rng.standard_normal(H, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    return x, w, b


def f32_linear_inputs(seq, N, K, seed=41):
    rng = np.random.default_rng(seed + seq + N + K)
    return (rng.standard_normal((seq, K), dtype=np.float32),
            (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.05)).astype(np.float32),
            rng.standard_normal(N, dtype=np.float32))


def dp_fixture_name(cfg, mask, variant):
    return f"dp_{cfg}_m{mask}" + (f"_{variant}" if variant else "") + ".npy"


def make_dp(digests):
    for cfg, shape_name, mask, variant in DP_CASES:
        with tempfile.TemporaryDirectory() as d:
            synth.write_dp_checkpoint(d, getattr(synth, shape_name), seed=0)
            digests["dp_" + cfg] = dir_digest(d)
            code = ("import sys,numpy as np; sys.path.insert(0, %r); from oracle import oracle; "
                    "from vla_simd_b200 import synth; r = oracle.reference(); sh = synth.%s; "
                    "import dataclasses; sh = dataclasses.replace(sh, num_inference_steps=%d); "
                    "f, s, n = synth.dp_inputs(sh, seed=1); "
                    "np.save(%r, r.dp_predict(%r, f, s, %s))") % (
                        ROOT, shape_name, getattr(synth, shape_name).num_inference_steps, os.path.join(HERE, dp_fixture_name(cfg, mask, variant)), d,
                        "None" if variant == "nonoise" else "n")
            env = dict(os.environ, DIFFUSION_INT8=str(mask), OMP_NUM_THREADS="1")
            if variant == "ddpm":
                env.update(DP_SCHEDULER="DDPM", DP_STEPS="10")
            subprocess.run([sys.executable, "-c", code], check=True, env=env)


# (config, shape, OCTO_INT8, variant): "" the seeded query of octo_inputs(seed=1),
# "nowrist" without the wrist camera, "pad" a 3-step window whose oldest step
# is history padding, "w1" a 1-step window, "seed" the reference's own noise
# draw from seed 7, "readout" the readout embedding instead of the actions
OCTO_CASES = [("small", "OCTO_SMALL", 63, ""), ("small", "OCTO_SMALL", 0, ""), ("small", "OCTO_SMALL", 63, "readout"),
              ("small", "OCTO_SMALL", 63, "nowrist"), ("small", "OCTO_SMALL", 63, "pad"),
              ("small", "OCTO_SMALL", 63, "w1"), ("small", "OCTO_SMALL", 63, "seed"),
              ("small", "OCTO_SMALL", 31, ""), ("base", "OCTO_BASELINE", 63, ""), ("erf", "OCTO_ERF", 63, "")]
# tokenizer cases: ids of each string under synth.octo_vocab()
T5_TEXTS = ["", " ", "pick up the red block", "PICK up \u00b2\u00bd \u2026 \ufb01", "a\tb\nc  d",
            "<extra_id_0> pick<extra_id_0>up", "x" * 40, "h\u00e9llo w\u00f6rld \u2603 \u65e5\u672c",
            "\x01\x7fab\u2581cd", "\uff21\uff22\uff23 fullwidth", "<unk> <pad> </s>"]


def octo_fixture_name(cfg, mask, variant):
    return f"octo_{cfg}_m{mask}" + (f"_{variant}" if variant else "") + ".npy"


def octo_query(shape, variant):
    """The inputs of one Octo fixture case: (primary, wrist, tmask, instruction, noise, z, seed)."""
    if variant == "pad":
        p, w, tm, ins, n, z = synth.octo_inputs(shape, seed=2, wnd=3)
        tm = np.array([0, 1, 1], np.uint8)
    elif variant == "w1":
        p, w, tm, ins, n, z = synth.octo_inputs(shape, seed=3, wnd=1)
    else:
        p, w, tm, ins, n, z = synth.octo_inputs(shape, seed=1)
    if variant == "nowrist":
        w = None
    if variant == "seed":
        n = z = None
    return p, w, tm, ins, n, z, 7


def make_octo(digests):
    for cfg, shape_name, mask, variant in OCTO_CASES:
        with tempfile.TemporaryDirectory() as d:
            shape = getattr(synth, shape_name)
            synth.write_octo_checkpoint(d, shape, seed=0)
            digests["octo_" + cfg] = dir_digest(d) + dir_digest(os.path.join(d, "tok"))[:16]
            call = ("r.octo_readout(d, d + '/tok', p, w, tm, ins, sh.d)" if variant == "readout"
                    else "r.octo_predict(d, d + '/tok', p, w, tm, ins, n, z, seed)")
            code = ("import sys,numpy as np; sys.path.insert(0, %r); sys.path.insert(0, %r); from oracle import oracle; "
                    "from vla_simd_b200 import synth; import make_golden as mg; r = oracle.reference(); "
                    "sh = synth.%s; d = %r; p, w, tm, ins, n, z, seed = mg.octo_query(sh, %r); "
                    "np.save(%r, %s)") % (ROOT, HERE, shape_name, d, variant,
                                          os.path.join(HERE, octo_fixture_name(cfg, mask, variant)), call)
            # the reference reads OCTO_INT8 once per process
            env = dict(os.environ, OCTO_INT8=str(mask), OMP_NUM_THREADS="1")
            subprocess.run([sys.executable, "-c", code], check=True, env=env)
    ref = oracle.reference()
    with tempfile.TemporaryDirectory() as d:
        synth.write_octo_checkpoint(d, synth.OCTO_SMALL, seed=0)
        ids = {t: ref.t5_tokenize(os.path.join(d, "tok"), t, 16).tolist() for t in T5_TEXTS}
        ids.update({synth.octo_instruction(i): ref.t5_tokenize(os.path.join(d, "tok"), synth.octo_instruction(i),
                                                               16).tolist() for i in range(20)})
    with open(os.path.join(HERE, "t5_ids.json"), "w") as f:
        json.dump(ids, f, indent=0, sort_keys=True)


# (config, shape, SMOLVLA_INT8, variant): "" the seeded query of smolvla_inputs(seed=1),
# "rtc" with real-time-chunking guidance, "seed" the reference's own noise draw
SMOLVLA_CASES = [("small", "SMOLVLA_SMALL", 63, ""), ("small", "SMOLVLA_SMALL", 0, ""),
                 ("small", "SMOLVLA_SMALL", 63, "rtc"), ("small", "SMOLVLA_SMALL", 63, "seed"),
                 ("small", "SMOLVLA_SMALL", 59, ""), ("base", "SMOLVLA_BASELINE", 63, ""),
                 ("edge", "SMOLVLA_EDGE", 63, "short"), ("edge", "SMOLVLA_EDGE", 0, "short")]


def smolvla_fixture_name(cfg, mask, variant):
    return f"smolvla_{cfg}_m{mask}" + (f"_{variant}" if variant else "") + ".npy"


def smolvla_query(shape, variant):
    """The inputs of one SmolVLA fixture case: (frames, instruction, state, noise,
    seed, prev, weights, max_guidance)."""
    frames, ins, state, noise = synth.smolvla_inputs(shape, seed=1)
    if variant == "short":   # fewer tokens than tok_maxlen: the rest are padding
        ins = "pick up"
    prev = weights = None
    mg = 0.0
    if variant == "rtc":
        rng = np.random.default_rng(21)
        prev = rng.standard_normal((3, shape.action_dim), dtype=np.float32)
        weights = rng.uniform(0.0, 1.0, shape.chunk).astype(np.float32)
        mg = 5.0
    if variant == "seed":
        noise = None
    return frames, ins, state, noise, 9, prev, weights, mg


def make_smolvla(digests):
    for cfg, shape_name, mask, variant in SMOLVLA_CASES:
        with tempfile.TemporaryDirectory() as d:
            shape = getattr(synth, shape_name)
            synth.write_smolvla_checkpoint(d, shape, seed=0)
            digests["smolvla_" + cfg] = dir_digest(d) + dir_digest(os.path.join(d, "tok"))[:16]
            code = ("import sys,numpy as np; sys.path.insert(0, %r); sys.path.insert(0, %r); from oracle import oracle; "
                    "from vla_simd_b200 import synth; import make_golden as mg; r = oracle.reference(); "
                    "sh = synth.%s; f, ins, st, nz, seed, pv, wt, g = mg.smolvla_query(sh, %r); "
                    "np.save(%r, r.smolvla_predict(%r, f, ins, st, nz, seed, pv, wt, g))") % (
                        ROOT, HERE, shape_name, variant, os.path.join(HERE, smolvla_fixture_name(cfg, mask, variant)),
                        d)
            env = dict(os.environ, SMOLVLA_INT8=str(mask), OMP_NUM_THREADS="1")
            subprocess.run([sys.executable, "-c", code], check=True, env=env)
    ref = oracle.reference()
    with tempfile.TemporaryDirectory() as d:
        synth.write_smolvla_checkpoint(d, synth.SMOLVLA_SMALL, seed=0)
        texts = T5_TEXTS + ["pick up the cube and place it in the bowl 3 times", "it's   done\n\n", "x1y22z333"]
        ids = {}
        for t in texts + [synth.octo_instruction(i) for i in range(20)]:
            tok, mask, n = ref.smolvla_tokenize(d, t)
            ids[t] = tok[:n].tolist()
    with open(os.path.join(HERE, "bpe_ids.json"), "w") as f:
        json.dump(ids, f, indent=0, sort_keys=True)


def main():
    ref = oracle.reference()
    if ref is None:
        sys.exit("oracle/_ref/libvla_ref.so missing: make -C oracle ref")
    digests = {}
    for flag, maker in (("--dp", make_dp), ("--octo", make_octo), ("--smolvla", make_smolvla)):   # one family only
        if flag in sys.argv:
            path = os.path.join(HERE, "checkpoints.json")
            digests = json.load(open(path))
            maker(digests)
            with open(path, "w") as f:
                json.dump(digests, f, indent=1, sort_keys=True)
            return
    make_dp(digests)
    make_octo(digests)
    make_smolvla(digests)
    for cfg, shape, mask in ACT_CASES:
        # the reference reads ACT_INT8 when it loads, so each mask runs in its own process
        with tempfile.TemporaryDirectory() as d:
            synth.write_act_checkpoint(d, shape, seed=0)
            digests[cfg] = dir_digest(d)
            code = ("import sys,numpy as np; sys.path.insert(0, %r); from oracle import oracle; "
                    "from vla_simd_b200 import synth; r = oracle.reference(); "
                    "f, s = synth.act_inputs(synth.%s, seed=1); "
                    "np.save(%r, r.act_predict(%r, f, s))") % (
                        ROOT, "ACT_SMALL" if cfg == "small" else "ACT_BASELINE",
                        os.path.join(HERE, f"act_{cfg}_m{mask}.npy"), d)
            env = dict(os.environ, ACT_INT8=str(mask))
            subprocess.run([sys.executable, "-c", code], check=True, env=env)
    with open(os.path.join(HERE, "checkpoints.json"), "w") as f:
        json.dump(digests, f, indent=1, sort_keys=True)

    arrays, meta = {}, {}
    for seq, N, K in GEMM_SHAPES:
        x, W, b = gemm_inputs(seq, N, K)
        xq, xs = ref.quantize_act_i8(x)
        panels, ws = ref.pack_weights_i8(W)
        out = ref.dense_linear_i8_ref(xq, xs, panels, ws, b, N, K)
        # int32 accumulators: the reference never exposes them; restate from its int8 operands
        wq = np.zeros((N, K), np.int8)
        Kp = ref.kpad(K)
        pan = panels[:N * Kp].reshape(N // 16, Kp // 4, 16, 4)
        wq[:, :] = pan.transpose(0, 2, 1, 3).reshape(N, Kp)[:, :K]
        acc = (xq[:, :K].astype(np.int64) @ wq.astype(np.int64).T).astype(np.int32)
        key = f"{seq}x{N}x{K}"
        meta[key] = {"xq": sha(xq[:, :K]), "ascale": sha(xs), "wq": sha(wq), "wscale": sha(ws), "acc": sha(acc),
                     "out": sha(out)}
        if seq * N <= 20000:
            arrays.update({f"{key}_xq": xq[:, :K], f"{key}_ascale": xs, f"{key}_acc": acc, f"{key}_out": out})
    fp = {}
    for sq, sk, nq, nkv in ATTN_CASES:
        Q, K, V = attn_inputs(sq, sk, nq, nkv)
        scale = np.float32(1.0) / np.sqrt(np.float32(64.0))
        fp[f"attn_{sq}x{sk}x{nq}x{nkv}"] = sha(ref.attention(Q, K, V, nq, nkv, 64, scale))
        fp[f"attn_causal_{sq}x{sk}x{nq}x{nkv}"] = sha(ref.attention(Q, K, V, nq, nkv, 64, scale,
                                                                    causal_mask(sq, sk)))
    for seq, H in LN_CASES:
        x, w, b = ln_inputs(seq, H)
        y = ref.layernorm(x, w, b, 1e-5)
        fp[f"ln_{seq}x{H}"] = sha(y)
        arrays[f"ln_{seq}x{H}"] = y
    for seq, N, K in F32_LINEAR_CASES:
        x, W, b = f32_linear_inputs(seq, N, K)
        fp[f"f32lin_{seq}x{N}x{K}"] = sha(ref.dense_linear(x, W, b))
    meta["fp32_ops"] = fp
    np.savez_compressed(os.path.join(HERE, "gemm.npz"), **arrays)
    with open(os.path.join(HERE, "gemm.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
