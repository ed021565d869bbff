"""The host byte-level BPE tokenizer SmolVLA's handles use (vla_bpe_tokenize)
against the reference's Tokenizer: the ids committed in
tests/golden/bpe_ids.json (made by the reference's vla_smolvla_tokenize, which
appends a newline and keeps the last tok_maxlen ids) and, when the reference
build is present, random strings compared live. No GPU needed."""
import json
import os

import numpy as np

from vla_simd_b200 import bpe_tokenize, synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _files(tmp_path):
    synth.smolvla_tokenizer_files(str(tmp_path / "tok"))
    voc = (tmp_path / "tok" / "vocab.txt").read_text(encoding="utf-8")
    mer = (tmp_path / "tok" / "merges.txt").read_text(encoding="utf-8")
    return voc, mer


def _as_handle(voc, mer, text, n):
    s = text
    while s.endswith("\n"):
        s = s[:-1]
    ids = bpe_tokenize(voc, mer, s + "\n")
    return ids[-n:] if len(ids) > n else ids


def test_bpe_matches_golden_ids(tmp_path):
    voc, mer = _files(tmp_path)
    ids = json.load(open(os.path.join(GOLDEN, "bpe_ids.json"), encoding="utf-8"))
    assert len(ids) > 20
    for s, want in ids.items():
        assert _as_handle(voc, mer, s, synth.SMOLVLA_SMALL.tok_maxlen).tolist() == want, repr(s)


def test_bpe_matches_reference_live(tmp_path, reference):
    d = synth.write_smolvla_checkpoint(str(tmp_path / "smol"), synth.SMOLVLA_SMALL, seed=0)
    voc = open(os.path.join(d, "tok", "vocab.txt"), encoding="utf-8").read()
    mer = open(os.path.join(d, "tok", "merges.txt"), encoding="utf-8").read()
    rng = np.random.default_rng(7)
    alphabet = list("abcdefghijklmnopqrstuvwxyz ABC.,!?'-\t\n0123456789") + [
        "é", "…", "½", "ａ", "日", "\x01", "  ", "'s", "'ll", "٣", "²", " "]
    for _ in range(120):
        s = "".join(rng.choice(alphabet, size=int(rng.integers(0, 40))))
        ids, mask, n = reference.smolvla_tokenize(d, s)
        assert np.array_equal(_as_handle(voc, mer, s, synth.SMOLVLA_SMALL.tok_maxlen), ids[:n]), repr(s)


def test_bpe_fuzz_matches_reference(tmp_path, reference):
    """Random Unicode text (no surrogates, no NUL) through the handle's
    tokenize path on both sides, 300 strings."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st
    d = synth.write_smolvla_checkpoint(str(tmp_path / "smol"), synth.SMOLVLA_SMALL, seed=0)
    voc = open(os.path.join(d, "tok", "vocab.txt"), encoding="utf-8").read()
    mer = open(os.path.join(d, "tok", "merges.txt"), encoding="utf-8").read()
    alphabet = st.characters(blacklist_categories=("Cs",), blacklist_characters="\x00")

    @settings(max_examples=300, deadline=None, suppress_health_check=list(HealthCheck), derandomize=True)
    @given(st.text(alphabet=alphabet, max_size=40))
    def check(s):
        ids, mask, n = reference.smolvla_tokenize(d, s)
        assert np.array_equal(_as_handle(voc, mer, s, synth.SMOLVLA_SMALL.tok_maxlen), ids[:n]), repr(s)

    check()


def test_bpe_split_rules_fuzz_matches_reference(tmp_path, reference):
    """Text drawn from the characters the split rules single out (ASCII and
    other whitespace, contraction letters after apostrophes, ASCII and other
    digits, letters and symbols of several scripts), 500 strings."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st
    d = synth.write_smolvla_checkpoint(str(tmp_path / "smol"), synth.SMOLVLA_SMALL, seed=0)
    voc = open(os.path.join(d, "tok", "vocab.txt"), encoding="utf-8").read()
    mer = open(os.path.join(d, "tok", "merges.txt"), encoding="utf-8").read()
    pieces = [" ", "  ", "\t", "\n", "\r\n", " ", "　", " ", "'", "'s", "'re", "'ve", "'ll", "'d",
              "'m", "'t", "'x", "0", "7", "42", "٣", "²", "５", "abc", "Robot", "été",
              "中文", "аб", "!", "?!", ".", "-", "_", "€", "\U0001f916", "pick", " up"]

    @settings(max_examples=500, deadline=None, suppress_health_check=list(HealthCheck), derandomize=True)
    @given(st.lists(st.sampled_from(pieces), max_size=24))
    def check(parts):
        s = "".join(parts)
        ids, mask, n = reference.smolvla_tokenize(d, s)
        assert np.array_equal(_as_handle(voc, mer, s, synth.SMOLVLA_SMALL.tok_maxlen), ids[:n]), repr(s)

    check()
