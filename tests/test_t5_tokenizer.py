"""The host T5 tokenizer Octo's handles use (vla_t5_tokenize) against the
reference's T5Tokenizer: the ids committed in tests/golden/t5_ids.json (made
by the reference through oracle/ref_octo_shim.cpp) and, when the reference
build is present, a wider set of strings compared live. No GPU needed."""
import json
import os

import numpy as np
import pytest

from vla_simd_b200 import synth, t5_tokenize

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _vocab_text():
    return "".join(f"{p}\t{sc!r}\n" for p, sc in synth.octo_vocab())


def test_tokenizer_matches_golden_ids():
    ids = json.load(open(os.path.join(GOLDEN, "t5_ids.json"), encoding="utf-8"))
    assert len(ids) > 20
    text = _vocab_text()
    for s, want in ids.items():
        assert t5_tokenize(text, s, 16).tolist() == want, repr(s)


def test_tokenizer_truncates_and_pads():
    text = _vocab_text()
    ids = t5_tokenize(text, "", 4)
    assert ids.tolist() == [1, 0, 0, 0]          # </s>, then <pad>
    ids = t5_tokenize(text, "ab " * 30, 8)
    assert ids[-1] == 1 and (ids[:-1] != 0).all()  # 7 pieces kept, then </s>


def test_tokenizer_matches_reference_live(tmp_path, reference):
    os.makedirs(tmp_path / "tok")
    (tmp_path / "tok" / "vocab.txt").write_text(_vocab_text(), encoding="utf-8")
    text = _vocab_text()
    rng = np.random.default_rng(3)
    alphabet = list("abcdefghijklmnopqrstuvwxyz ABC.,!?'-\t") + ["é", "…", "½", "ａ", "▁",
                                                                    "日", "\x01", "<extra_id_0>", "<pad>"]
    cases = ["".join(rng.choice(alphabet, size=int(rng.integers(0, 30)))) for _ in range(200)]
    for s in cases:
        for n in (4, 16):
            assert np.array_equal(t5_tokenize(text, s, n), reference.t5_tokenize(str(tmp_path / "tok"), s, n)), repr(s)


def test_tokenizer_fuzz_matches_reference(tmp_path, reference):
    """Random Unicode text (no surrogates, no NUL), both tokenizers, 300 strings."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st
    os.makedirs(tmp_path / "tok", exist_ok=True)
    (tmp_path / "tok" / "vocab.txt").write_text(_vocab_text(), encoding="utf-8")
    text = _vocab_text()
    tok_dir = str(tmp_path / "tok")
    alphabet = st.characters(blacklist_categories=("Cs",), blacklist_characters="\x00")

    @settings(max_examples=300, deadline=None, suppress_health_check=list(HealthCheck), derandomize=True)
    @given(st.text(alphabet=alphabet, max_size=40))
    def check(s):
        assert np.array_equal(t5_tokenize(text, s, 16), reference.t5_tokenize(tok_dir, s, 16)), repr(s)

    check()
