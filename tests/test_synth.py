"""Synthetic-data pipeline with a scripted LLM (no network): taxonomy, quality gate,
dedup, grounded chunking, sharding, fenced resume."""

import json
import re

import pytest

from pluggy_b200.synth.dedup import Deduper
from pluggy_b200.synth.grounded import load_chunks
from pluggy_b200.synth.judge import evaluate
from pluggy_b200.synth.llm import ScriptedClient, _parse_json, build_client
from pluggy_b200.synth.pipeline import run_pipeline
from pluggy_b200.synth.writer import ShardWriter


def _words(seed: str, n: int = 120) -> str:
    import hashlib

    out = []
    h = seed.encode()
    for _ in range(n):
        h = hashlib.sha1(h).digest()
        out.append("w" + h.hex()[:6])
    return " ".join(out)


def scripted(score_for=lambda doc: 8, dup_every: int = 0):
    """Taxonomy -> two topics per domain; documents -> unique text per prompt;
    judge -> ``score_for(doc)``; rewrite -> the document with 'REFINED' prepended."""
    n = {"docs": 0}

    def fn(prompt, system, max_tokens):
        if "Break the field" in prompt:
            d = re.search(r'field "([^"]+)"', prompt).group(1)
            return json.dumps({"topics": [{"topic": f"{d} part {i}", "summary": "s"}
                                          for i in range(2)]})
        if prompt.startswith("Rate the document"):
            doc = prompt.split("<document>\n", 1)[1].rsplit("\n</document>", 1)[0]
            return "```json\n" + json.dumps({"score": score_for(doc), "weaknesses": "thin"}) + "\n```"
        if prompt.startswith("Rewrite this document"):
            doc = prompt.split("<document>\n", 1)[1].rsplit("\n</document>", 1)[0]
            return "REFINED " + doc
        n["docs"] += 1
        if dup_every and n["docs"] % dup_every == 0:
            return _words("the same text every time")
        return _words(prompt)

    return ScriptedClient(fn)


def _cfg(tmp_path, **kw):
    c = {"model": "grok-4", "seed": 0, "seed_domains": ["physics", "history"],
         "taxonomy": {"subtopics_per_domain": 2},
         "generation": {"docs_per_topic": 3, "concurrency": 4},
         "quality": {"enabled": True, "min_score": 7, "refine_min": 5, "max_refine_rounds": 1},
         "dedup": {"ngram": 13, "jaccard_threshold": 0.8},
         "output": {"dir": str(tmp_path / "out"), "shard_docs": 5}}
    c.update(kw)
    return c


def _rows(d):
    rows = []
    for p in sorted(d.glob("shard-*.jsonl")):
        rows += [json.loads(x) for x in p.read_text().splitlines()]
    return rows


def test_parse_json_and_provider():
    assert _parse_json('sure: {"a": 1} done') == {"a": 1}
    assert _parse_json("```json\n{\"a\": 2}\n```") == {"a": 2}
    assert _parse_json("nothing") is None
    assert type(build_client({"model": "grok-4"})).__name__ == "GrokClient"
    assert type(build_client({"model": "claude-x"})).__name__ == "AnthropicClient"
    with pytest.raises(ValueError):
        build_client({"provider": "other"})


def test_quality_gate():
    doc = _words("d")
    assert evaluate(scripted(lambda d: 9), doc, {}, 100) == (doc, 9)
    assert evaluate(scripted(lambda d: 3), doc, {}, 100) == (None, None)  # below refine band
    # in the refine band: rewritten, re-judged, kept when it passes
    out, s = evaluate(scripted(lambda d: 8 if d.startswith("REFINED") else 6), doc, {}, 100)
    assert out.startswith("REFINED") and s == 8
    # still below min_score after the allowed rewrites: dropped
    assert evaluate(scripted(lambda d: 6), doc, {"max_refine_rounds": 2}, 100) == (None, None)
    # out-of-range judge scores are failures
    assert evaluate(scripted(lambda d: 11), doc, {}, 100) == (None, None)


def test_dedup_near_and_exact():
    d = Deduper(ngram=5, threshold=0.8)
    a = _words("a", 400)
    assert not d.is_duplicate(a)
    assert d.is_duplicate(a.upper())  # exact after normalisation
    near = a.split()
    near[200] = "changed"
    assert d.is_duplicate(" ".join(near))  # one word changed: Jaccard ~0.98
    assert not d.is_duplicate(_words("b", 400))
    half = a.split()[:200] + _words("c", 200).split()
    assert not d.is_duplicate(" ".join(half))  # Jaccard ~1/3


def test_load_chunks(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    (src / "a.jsonl").write_text(json.dumps({"text": " ".join(f"x{i}" for i in range(260))}) + "\n")
    (src / "b.jsonl").write_text(json.dumps({"text": " ".join(f"y{i}" for i in range(110))}) + "\n")
    ch = load_chunks(src, 100)
    # a: 100, 100, 60 (kept, >= 25); b: 100, 10 (dropped, < 25)
    assert [len(c.split()) for c in ch] == [100, 100, 60, 100]
    with pytest.raises(FileNotFoundError):
        load_chunks(tmp_path / "empty", 100)


def test_writer_tmp_rename_and_numbering(tmp_path):
    w = ShardWriter(tmp_path, shard_docs=2)
    for i in range(5):
        w.add({"text": str(i)})
    w.close({"x": 1})
    assert sorted(p.name for p in tmp_path.glob("shard-*")) == [
        "shard-00000.jsonl", "shard-00001.jsonl", "shard-00002.jsonl"]
    assert json.loads((tmp_path / "manifest.json").read_text())["num_shards"] == 3
    w2 = ShardWriter(tmp_path, shard_docs=2)
    assert w2.shard_idx == 3
    assert not list(tmp_path.glob("*.tmp"))


def test_pipeline_topics_grounded_and_dupes(tmp_path):
    src = tmp_path / "uploads"
    src.mkdir()
    (src / "u.jsonl").write_text("\n".join(json.dumps({"text": _words(f"u{i}", 150)})
                                           for i in range(3)) + "\n")
    cfg = _cfg(tmp_path, grounding={"dir": str(src), "chunk_words": 100, "gens_per_chunk": 2})
    res = run_pipeline(cfg, client=scripted(dup_every=4), log=lambda *_: None)
    rows = _rows(tmp_path / "out")
    n_jobs = 2 * 2 * 3 + 6 * 2  # topics x docs + chunks (3 docs x 2 windows) x gens
    assert res["kept"] + res["dupes"] + res["dropped"] == n_jobs
    assert res["dupes"] >= 1 and len(rows) == res["kept"]
    topic_rows = [r for r in rows if "topic" in r]
    grounded = [r for r in rows if "chunk_id" in r]
    assert topic_rows and grounded
    assert set(topic_rows[0]) == {"text", "domain", "topic", "style", "score"}
    assert set(grounded[0]) == {"text", "source", "chunk_id", "mode", "score"}
    st = json.loads((tmp_path / "out" / "state.json").read_text())
    assert len(st["done"]) == n_jobs and st["num_chunks"] == 6
    assert json.loads((tmp_path / "out" / "manifest.json").read_text())["kept"] == res["kept"]
    # changed uploads under the same output dir are refused
    (src / "v.jsonl").write_text(json.dumps({"text": _words("v", 150)}) + "\n")
    with pytest.raises(ValueError, match="fresh output dir"):
        run_pipeline(cfg, client=scripted(), log=lambda *_: None)


def test_pipeline_fenced_resume(tmp_path):
    """A crash after some shards: only keys whose documents reached a shard are done;
    the resumed run writes exactly the rest, with no duplicates."""
    cfg = _cfg(tmp_path, generation={"docs_per_topic": 5, "concurrency": 1})
    calls = {"n": 0}
    base = scripted()

    def crashing(prompt, system, max_tokens):
        if not prompt.startswith(("Break", "Rate", "Rewrite")):
            calls["n"] += 1
            if calls["n"] == 13:
                raise RuntimeError("worker died")
        return base.fn(prompt, system, max_tokens)

    with pytest.raises(RuntimeError):
        run_pipeline(cfg, client=ScriptedClient(crashing), log=lambda *_: None)
    out = tmp_path / "out"
    st = json.loads((out / "state.json").read_text())
    rows = _rows(out)
    assert len(rows) == 10 and len(st["done"]) == 10  # two full shards fenced, the rest not
    topics_before = st["topics"]
    res = run_pipeline(cfg, client=scripted(), log=lambda *_: None)
    st = json.loads((out / "state.json").read_text())
    rows = _rows(out)
    assert st["topics"] == topics_before  # taxonomy pinned
    assert res["kept"] == 10 and len(rows) == 20 and len(st["done"]) == 20
    assert len({r["text"] for r in rows}) == 20


def test_no_work_is_an_error(tmp_path):
    with pytest.raises(ValueError, match="no work"):
        run_pipeline({"output": {"dir": str(tmp_path)}}, client=scripted())
