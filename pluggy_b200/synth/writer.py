"""Sharded JSONL output, each shard written to a temporary name and renamed.

Parity: reference ``pluggy/synth/writer.py:18-53``: ``shard-NNNNN.jsonl`` files of
``shard_docs`` rows, numbering continued after the shards already present, and a
``manifest.json`` on close. A killed run leaves at most a ``.tmp`` file, never a
partial shard.
"""

from __future__ import annotations

import json
import os
from pathlib import Path


class ShardWriter:
    def __init__(self, out_dir, shard_docs: int = 1000):
        self.dir = Path(out_dir)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.shard_docs = shard_docs
        self.rows: list[dict] = []
        self.total = 0
        self.shard_idx = len(list(self.dir.glob("shard-*.jsonl")))

    def add(self, row: dict) -> None:
        self.rows.append(row)
        self.total += 1
        if len(self.rows) >= self.shard_docs:
            self.flush()

    def flush(self) -> None:
        if not self.rows:
            return
        final = self.dir / f"shard-{self.shard_idx:05d}.jsonl"
        tmp = final.with_name(final.name + ".tmp")
        with open(tmp, "w", encoding="utf-8") as f:
            f.writelines(json.dumps(r, ensure_ascii=False) + "\n" for r in self.rows)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, final)
        self.shard_idx += 1
        self.rows = []

    def close(self, manifest_extra: dict | None = None) -> None:
        self.flush()
        man = {"num_shards": self.shard_idx, "docs_written_this_run": self.total}
        man.update(manifest_extra or {})
        tmp = self.dir / "manifest.json.tmp"
        with open(tmp, "w") as f:
            json.dump(man, f, indent=2)
        os.replace(tmp, self.dir / "manifest.json")
