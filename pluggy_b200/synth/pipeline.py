"""Synthetic pretraining data: taxonomy -> (generate -> judge -> refine) -> dedup -> shards.

Parity: reference ``pluggy/synth/pipeline.py:83-212`` (``run_pipeline``).

* Work is a list of jobs with stable keys: ``"{topic_id}:{style}:{k}"`` for topic
  documents and ``"g{chunk}:{mode}:{k}"`` for grounded ones. The list is shuffled
  with the config seed so a partial run covers topics evenly.
* LLM calls run on a thread pool (``generation.concurrency`` workers); dedup and the
  shard writer run only on the calling thread, so they need no locks.
* ``state.json`` pins the taxonomy (so topic ids are stable), the grounded chunk
  count (a resume with different uploads is refused) and the finished job keys. A
  key is committed only once the shard holding its document is on disk: the same
  fencing the checkpointer uses, so a crash never loses a document whose key was
  recorded, and never records a key whose document was lost.
* The deduper is seeded from shards already written, so a resumed run dedups
  against earlier output.
"""

from __future__ import annotations

import json
import os
import random
from concurrent.futures import ThreadPoolExecutor, as_completed
from pathlib import Path

from pluggy_b200.synth.dedup import Deduper
from pluggy_b200.synth.generate import STYLES, generate_doc
from pluggy_b200.synth.grounded import GROUNDED_MODES, generate_grounded, load_chunks
from pluggy_b200.synth.judge import evaluate
from pluggy_b200.synth.llm import build_client
from pluggy_b200.synth.taxonomy import build_taxonomy
from pluggy_b200.synth.writer import ShardWriter


def load_state(path: Path) -> dict:
    if path.exists():
        with open(path) as f:
            return json.load(f)
    return {"topics": None, "done": []}


def save_state(path: Path, state: dict) -> None:
    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "w") as f:
        json.dump(state, f)
    os.replace(tmp, path)


def run_job(client, job: dict, gen_cfg: dict, quality_cfg: dict):
    """One document: generate, then the quality gate. Returns ``(job, doc|None, score)``."""
    max_tokens = gen_cfg.get("max_tokens", 4096)
    if job["kind"] == "topic":
        doc = generate_doc(client, job["topic"], job["style"], job["variant"], max_tokens)
        source = None
    else:
        doc = generate_grounded(client, job["chunk"], job["mode"], job["variant"], max_tokens)
        source = job["chunk"]
    if doc is None or not quality_cfg.get("enabled", True):
        return job, doc, None
    doc, score = evaluate(client, doc, quality_cfg, max_tokens, source=source)
    return job, doc, score


def make_row(job: dict, doc: str, score, grounding_cfg) -> dict:
    """The loader reads ``text``; the other columns are provenance."""
    if job["kind"] == "topic":
        return {"text": doc, "domain": job["topic"]["domain"], "topic": job["topic"]["topic"],
                "style": job["style"], "score": score}
    return {"text": doc, "source": grounding_cfg["dir"], "chunk_id": job["chunk_id"],
            "mode": job["mode"], "score": score}


def plan_jobs(cfg: dict, state: dict, state_path: Path, client) -> tuple[list[dict], int]:
    done = set(state["done"])
    if state["topics"] is None:
        domains = cfg.get("seed_domains") or []
        n = cfg.get("taxonomy", {}).get("subtopics_per_domain", 10)
        state["topics"] = build_taxonomy(client, domains, n) if domains else []
        save_state(state_path, state)
    gen = cfg.get("generation", {})
    styles = gen.get("styles") or list(STYLES)
    jobs = []
    for t in state["topics"]:
        for k in range(gen.get("docs_per_topic", 2)):
            style = styles[k % len(styles)]
            key = f"{t['id']}:{style}:{k}"
            if key not in done:
                jobs.append({"kind": "topic", "key": key, "topic": t, "style": style, "variant": k})
    nchunks = 0
    g = cfg.get("grounding")
    if g:
        chunks = load_chunks(g["dir"], g.get("chunk_words", 600))
        nchunks = len(chunks)
        if state.get("num_chunks") is None:
            state["num_chunks"] = nchunks
            save_state(state_path, state)
        if state["num_chunks"] != nchunks:
            raise ValueError(
                f"the grounding source now yields {nchunks} chunks but this output was started "
                f"with {state['num_chunks']}; resuming would ground job keys on different text. "
                "Write changed uploads to a fresh output dir.")
        modes = g.get("modes") or list(GROUNDED_MODES)
        for ci, chunk in enumerate(chunks):
            for k in range(g.get("gens_per_chunk", 1)):
                mode = modes[k % len(modes)]
                key = f"g{ci}:{mode}:{k}"
                if key not in done:
                    jobs.append({"kind": "grounded", "key": key, "chunk": chunk, "chunk_id": ci,
                                 "mode": mode, "variant": k})
    random.Random(cfg.get("seed", 0)).shuffle(jobs)
    return jobs, nchunks


def run_pipeline(cfg: dict, client=None, log=print) -> dict:
    if not (cfg.get("seed_domains") or cfg.get("grounding")):
        raise ValueError("the config produces no work: set seed_domains (topic documents), "
                         "grounding (documents from uploaded text), or both")
    client = client if client is not None else build_client(cfg)
    out = Path(cfg["output"]["dir"])
    out.mkdir(parents=True, exist_ok=True)
    state_path = out / "state.json"
    state = load_state(state_path)
    jobs, nchunks = plan_jobs(cfg, state, state_path, client)
    done = set(state["done"])
    log(f"synth: {len(state['topics'])} topics, {nchunks} grounded chunks, {len(jobs)} documents "
        f"to write ({len(done)} already done)")

    dd = cfg.get("dedup", {})
    dedup = Deduper(ngram=dd.get("ngram", 13), threshold=dd.get("jaccard_threshold", 0.8))
    for shard in sorted(out.glob("shard-*.jsonl")):
        with open(shard, encoding="utf-8") as f:
            for line in f:
                dedup.is_duplicate(json.loads(line)["text"])

    writer = ShardWriter(out, cfg["output"].get("shard_docs", 1000))
    counts = {"kept": 0, "dropped": 0, "dupes": 0}
    unfenced: list[str] = []
    fence = writer.shard_idx

    def commit(force: bool = False) -> None:
        nonlocal fence
        if force or writer.shard_idx > fence:
            done.update(unfenced)
            unfenced.clear()
            state["done"] = sorted(done)
            fence = writer.shard_idx
            save_state(state_path, state)

    gen, quality = cfg.get("generation", {}), cfg.get("quality", {})
    pool = ThreadPoolExecutor(max_workers=gen.get("concurrency", 8))
    try:
        futs = [pool.submit(run_job, client, j, gen, quality) for j in jobs]
        for i, fut in enumerate(as_completed(futs), 1):
            job, doc, score = fut.result()
            if doc is None:
                counts["dropped"] += 1
            elif dedup.is_duplicate(doc):
                counts["dupes"] += 1
            else:
                writer.add(make_row(job, doc, score, cfg.get("grounding")))
                counts["kept"] += 1
            unfenced.append(job["key"])
            commit()
            if i % 25 == 0:
                log(f"synth: {i}/{len(jobs)} jobs, {counts['kept']} kept / "
                    f"{counts['dropped']} dropped / {counts['dupes']} dupes")
    finally:
        # on an error, queued jobs are cancelled; the keys fenced so far stay valid
        pool.shutdown(wait=True, cancel_futures=True)
    writer.close(manifest_extra={"model": cfg.get("model", "grok-4"), **counts})
    commit(force=True)
    log(f"synth: done, {counts['kept']} kept, {counts['dropped']} dropped, {counts['dupes']} dupes "
        f"-> {writer.shard_idx} shards in {out}")
    return counts
