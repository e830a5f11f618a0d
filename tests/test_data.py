"""Dataloader: packers, source resolution, mixing shares, exact resume, synthetic rows."""

import json

import numpy as np
import pytest
import torch

from pluggy_b200.dataloader.builder import build_dataloader, resolve_sources
from pluggy_b200.dataloader.packers import ListPacker, ListPackerBestFit, NumpyPacker, TensorPacker
from pluggy_b200.dataloader.synthetic import SyntheticBatches, SyntheticZipfRows

EOS, PAD = 1, 0


class _Enc:
    def __init__(self, ids):
        self.ids = ids


class FakeTokenizer:
    """Text of space-separated integers -> those integers (no vocab, no network)."""

    def encode_batch(self, texts):
        return [_Enc([int(w) for w in t.split()]) for t in texts]

    def token_to_id(self, tok):
        return {"<eos>": EOS, "<pad>": PAD}.get(tok)


def _docs(seed=0, n=60, lo=1, hi=300):
    rng = np.random.default_rng(seed)
    return [list(rng.integers(2, 1000, int(rng.integers(lo, hi)))) for _ in range(n)]


def test_stream_packers_identical():
    docs = _docs()
    rows = [P(FakeTokenizer(), 64, EOS).pack(docs) for P in (ListPacker, NumpyPacker, TensorPacker)]
    assert rows[0] == rows[1] == rows[2]
    stream = [t for d in docs for t in d + [EOS]]
    assert sum(rows[0], []) == stream[: len(rows[0]) * 64]  # contiguous, tail dropped
    for P in (ListPacker, NumpyPacker, TensorPacker):
        assert P(FakeTokenizer(), 64, EOS).pack([]) == []
        assert P(FakeTokenizer(), 64, EOS).pack_to_tensor([]).shape == (0, 64)


def test_bestfit_conserves_tokens():
    docs = _docs(1, 80, 1, 200)
    rows = ListPackerBestFit(FakeTokenizer(), 64, EOS, PAD).pack(docs)
    assert all(len(r) == 64 for r in rows)
    got = sorted(t for r in rows for t in r if t not in (EOS, PAD))
    want = sorted(t for d in docs for t in d)
    assert got == want  # every content token lands in exactly one row
    assert sum(r.count(EOS) for r in rows) == len(docs)
    # padding only fills the end of a bin
    for r in rows:
        if PAD in r:
            i = r.index(PAD)
            assert set(r[i:]) == {PAD}
    # fewer rows than the stream packer would need for the same tokens without cuts
    assert len(rows) <= -(-sum(len(d) + 1 for d in docs) // 64) + 8
    assert ListPackerBestFit(FakeTokenizer(), 64, EOS).pack([]) == []


def test_resolve_sources_rules():
    one = resolve_sources({"data_files": "a.jsonl", "text_field": "text"})
    assert len(one) == 1 and one[0]["weight"] == 1.0 and one[0]["split"] == "train"
    two = resolve_sources({"text_field": "body", "sources": [
        {"data_files": "a.jsonl", "weight": 3}, {"data_files": "b.jsonl", "weight": 1, "text_field": "t"}]})
    assert [s["weight"] for s in two] == [0.75, 0.25]
    assert [s["text_field"] for s in two] == ["body", "t"]  # inherited vs own
    with pytest.raises(AssertionError, match="weight"):
        resolve_sources({"text_field": "x", "sources": [{"data_files": "a"}, {"data_files": "b"}]})
    with pytest.raises(AssertionError, match="unknown"):
        resolve_sources({"sources": [{"data_files": "a", "text_field": "x", "colour": 1}]})
    with pytest.raises(AssertionError, match="exactly one"):
        resolve_sources({"sources": [{"data_files": "a", "name": "b", "text_field": "x"}]})


def _write_source(path, marker, n_docs, words):
    with open(path, "w") as f:
        for i in range(n_docs):
            f.write(json.dumps({"text": " ".join([str(marker)] * words), "i": i}) + "\n")


def _cfg(tmp_path, **kw):
    a, b = tmp_path / "a.jsonl", tmp_path / "b.jsonl"
    _write_source(a, 7, 4000, 31)
    _write_source(b, 9, 4000, 31)
    c = {"sources": [{"data_files": str(a), "weight": 0.75}, {"data_files": str(b), "weight": 0.25}],
         "text_field": "text", "eos_token": "<eos>", "pad_token": "<pad>", "seq_len": 32,
         "micro_batch_size": 8, "num_workers": 0, "seed": 0, "shuffle_buffer": 100, "pack_batch": 50}
    c.update(kw)
    return c


def test_mixing_token_shares_and_row_purity(tmp_path):
    dl = build_dataloader(_cfg(tmp_path), FakeTokenizer(), -100, 0, 1)
    counts = {7: 0, 9: 0}
    it = iter(dl)
    for _ in range(100):
        ids = next(it)["input_ids"]
        for row in ids.tolist():
            content = {t for t in row if t != EOS}
            assert len(content) == 1  # a row never mixes sources
            counts[content.pop()] += 1
    share = counts[7] / (counts[7] + counts[9])
    assert abs(share - 0.75) < 0.05, share


@pytest.mark.parametrize("workers", [0, 2])
def test_loader_resume_replays_same_rows(tmp_path, workers):
    cfg = _cfg(tmp_path, num_workers=workers)
    dl = build_dataloader(cfg, FakeTokenizer(), -100, 0, 1)
    it = iter(dl)
    for _ in range(5):
        next(it)
    state = dl.state_dict()
    want = [next(it)["input_ids"] for _ in range(4)]
    dl2 = build_dataloader(cfg, FakeTokenizer(), -100, 0, 1)
    dl2.load_state_dict(state)
    it2 = iter(dl2)
    got = [next(it2)["input_ids"] for _ in range(4)]
    for g, w in zip(got, want):
        assert torch.equal(g, w)


def test_per_rank_streams_differ(tmp_path):
    cfg = _cfg(tmp_path)
    r0 = next(iter(build_dataloader(cfg, FakeTokenizer(), -100, 0, 2)))["input_ids"]
    r1 = next(iter(build_dataloader(cfg, FakeTokenizer(), -100, 1, 2)))["input_ids"]
    assert not torch.equal(r0, r1)


def test_synthetic_zipf_rows():
    src = SyntheticZipfRows(vocab_size=1000, seq_len=8192, eos_id=999, seed=3, min_doc=512,
                            max_doc=4096)
    r = src.row(5)
    assert np.array_equal(r, src.row(5))  # regenerated from the index alone
    eos = np.flatnonzero(r == 999)
    gaps = np.diff(eos)
    assert len(eos) >= 1 and gaps.min() >= 512 and gaps.max() <= 4096
    counts = np.bincount(np.concatenate([src.row(i) for i in range(8)]), minlength=1000)
    assert counts[0] > counts[1] > counts[10] > counts[100]  # Zipf-ranked
    other = SyntheticZipfRows(vocab_size=1000, seq_len=8192, eos_id=999, seed=3, dp_rank=1)
    assert not np.array_equal(other.row(5), r)
    uni = SyntheticZipfRows(vocab_size=8192, seq_len=256, seed=0, kind="uniform").row(0)
    assert uni.min() >= 0 and uni.max() < 8192 and len(np.unique(uni)) > 200


def test_synthetic_batches_resume():
    src = SyntheticZipfRows(vocab_size=500, seq_len=64, seed=1)
    b = SyntheticBatches(src, 4)
    for _ in range(3):
        next(b)
    st = b.state_dict()
    want = next(b)["input_ids"]
    b2 = SyntheticBatches(SyntheticZipfRows(vocab_size=500, seq_len=64, seed=1), 4)
    b2.load_state_dict(st)
    assert torch.equal(next(b2)["input_ids"], want)
