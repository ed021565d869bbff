"""vla.simd GGUF checkpoints (the container the reference's converters write):
synth.pack_gguf packs a converted directory the way the reference's reader
expects (src/io/gguf_vla_simd.cpp), checked by loading it with the reference
itself: the same actions as from the directory."""
import os

import numpy as np

from vla_simd_b200 import synth


def test_reference_reads_packed_act_gguf(tmp_path, reference, monkeypatch):
    monkeypatch.setenv("ACT_INT8", "63")
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_SMALL, seed=0)
    g = synth.pack_gguf(d, str(tmp_path / "act.gguf"), "act")
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    assert np.array_equal(reference.act_predict(d, f, s), reference.act_predict(g, f, s))


def test_reference_reads_packed_dp_gguf(tmp_path, reference, monkeypatch):
    monkeypatch.setenv("DIFFUSION_INT8", "3")
    d = synth.write_dp_checkpoint(str(tmp_path / "dp"), synth.DP_SMALL, seed=0)
    os.makedirs(tmp_path / "only")
    g = synth.pack_gguf(d, str(tmp_path / "only" / "dp.gguf"), "diffusion")
    f, s, n = synth.dp_inputs(synth.DP_SMALL, seed=1)
    want = reference.dp_predict(d, f, s, n)
    assert np.array_equal(want, reference.dp_predict(g, f, s, n))
    # a directory holding exactly one .gguf and no .meta mounts that file
    assert np.array_equal(want, reference.dp_predict(str(tmp_path / "only"), f, s, n))


def test_packed_gguf_layout(tmp_path):
    import struct
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_SMALL, seed=0)
    g = synth.pack_gguf(d, str(tmp_path / "act.gguf"), "act")
    raw = open(g, "rb").read()
    assert raw[:4] == b"GGUF" and struct.unpack_from("<I", raw, 4)[0] == 3
    n_tensors, n_kv = struct.unpack_from("<QQ", raw, 8)
    assert n_tensors == 3          # backbone.bin, act.bin, stats.bin
    assert n_kv == 5 + 3           # general / vla_simd keys + config.txt, backbone.meta, act.meta
