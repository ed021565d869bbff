"""The library's GGUF mount on the B200: a vla.simd GGUF (file path, or a
directory holding only it) loads to the same bits as the converted directory
it was packed from; a GGUF of another architecture is refused."""
import os
import struct

import numpy as np
import pytest

from vla_simd_b200 import synth

pytestmark = pytest.mark.gpu


def test_act_gguf_equals_directory(tmp_path, monkeypatch):
    from vla_simd_b200 import ActPolicy
    monkeypatch.setenv("ACT_INT8", "63")
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_SMALL, seed=0)
    g = synth.pack_gguf(d, str(tmp_path / "act.gguf"), "act")
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    a = ActPolicy(d)
    want = a.predict(f, s)
    a.close()
    b = ActPolicy(g)
    assert np.array_equal(b.predict(f, s), want)
    b.close()
    assert np.array_equal(want, np.load(os.path.join(os.path.dirname(__file__), "golden", "act_small_m63.npy")))


def test_dp_gguf_directory_mount_equals_directory(tmp_path, monkeypatch):
    from vla_simd_b200 import DiffusionPolicy
    monkeypatch.setenv("DIFFUSION_INT8", "3")
    d = synth.write_dp_checkpoint(str(tmp_path / "dp"), synth.DP_SMALL, seed=0)
    os.makedirs(tmp_path / "only")
    synth.pack_gguf(d, str(tmp_path / "only" / "dp.gguf"), "diffusion")
    f, s, n = synth.dp_inputs(synth.DP_SMALL, seed=1)
    a = DiffusionPolicy(d)
    want = a.predict(f, s, n)
    a.close()
    b = DiffusionPolicy(str(tmp_path / "only"))
    assert np.array_equal(b.predict(f, s, n), want)
    b.close()


def test_foreign_gguf_is_refused(tmp_path, monkeypatch):
    from vla_simd_b200 import ActPolicy
    monkeypatch.setenv("ACT_INT8", "63")
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_SMALL, seed=0)
    g = synth.pack_gguf(d, str(tmp_path / "act.gguf"), "act")
    raw = bytearray(open(g, "rb").read())
    i = raw.index(b"vla-simd")
    raw[i:i + 8] = b"smolvla\0"[:8]           # another architecture, same length
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError):
        ActPolicy(str(bad))
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(bytes(raw[:100]))
    with pytest.raises(RuntimeError):
        ActPolicy(str(trunc))
