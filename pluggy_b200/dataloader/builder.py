"""Dataloader construction: source resolution, per-source packing, token mixing.

Parity: reference ``pluggy/dataloader/builder.py:68-371``:

* ``resolve_sources``: one schema for single-dataset and ``sources[]`` configs;
  per-source keys inherit from the top level; unknown keys, a missing
  ``text_field``, both/neither of ``name``/``data_files`` and weightless mixture
  members are rejected; weights are normalised to token fractions;
* each source is loaded (HF streaming, or local jsonl), its text column renamed
  to ``text``, shuffled, split by dp rank and packed BEFORE mixing, so every row
  is ``seq_len`` real tokens and mixture weights are token shares;
* ``mix_streams`` interleaves with ``mixing_seed = seed + 10000 + dp_rank``;
* a ``StatefulDataLoader`` with pinned memory yields micro-batches.

Addition: ``data.synthetic`` (``{"kind": "zipf", "s": 1.1, "min_doc": 512,
"max_doc": 4096}``) builds the offline synthetic source used by the benchmarks.
"""

from __future__ import annotations

import torch

from pluggy_b200.dataloader.packers import ListPacker

SOURCE_KEYS = ("name", "data_files", "config", "split", "text_field", "weight",
               "shuffle_buffer", "pack_batch")
STOPPING_STRATEGIES = ("first_exhausted", "all_exhausted", "all_exhausted_without_replacement")


class Collator:
    def __init__(self, tokenizer, ignore_index: int):
        self.tokenizer = tokenizer
        self.ignore_index = ignore_index

    def __call__(self, examples):
        ids = torch.tensor([ex["input_ids"] for ex in examples], dtype=torch.long)
        return {"input_ids": ids, "labels": ids.clone()}


def normalize_weights(weights: list[float]) -> list[float]:
    total = sum(weights)
    assert total > 0, f"data source weights must sum to something positive, got {weights}"
    return [w / total for w in weights]


def resolve_sources(data_cfg: dict) -> list[dict]:
    sources = data_cfg.get("sources")
    if sources is None:
        sources = [{k: data_cfg[k] for k in SOURCE_KEYS if k in data_cfg}]
    assert sources, "data.sources is empty: give it at least one dataset"
    out = []
    for i, src in enumerate(sources):
        unknown = set(src) - set(SOURCE_KEYS)
        assert not unknown, (
            f"data.sources[{i}] has unknown key(s) {sorted(unknown)}; a source may set "
            f"{list(SOURCE_KEYS)}"
        )
        assert ("name" in src) != ("data_files" in src), (
            f"data.sources[{i}] must have exactly one of 'name' or 'data_files'"
        )
        label = src.get("name") or src["data_files"]

        def inh(key, default=None, _src=src):
            return _src.get(key, data_cfg.get(key, default))

        text_field = inh("text_field")
        assert text_field is not None, f"data.sources[{i}] ({label}) has no 'text_field'"
        weight = src.get("weight", 1.0 if len(sources) == 1 else None)
        assert weight is not None, f"data.sources[{i}] ({label}) has no 'weight'"
        assert weight > 0, f"data.sources[{i}] ({label}) has non-positive weight {weight}"
        out.append({
            "name": src.get("name"), "data_files": src.get("data_files"), "label": label,
            "config": inh("config"), "split": inh("split", "train"), "text_field": text_field,
            "weight": weight, "shuffle_buffer": inh("shuffle_buffer"),
            "pack_batch": inh("pack_batch", 1000),
        })
    for s, w in zip(out, normalize_weights([s["weight"] for s in out]), strict=True):
        s["weight"] = w
    return out


def load_source(src):
    import datasets

    if src["data_files"] is not None:
        return datasets.load_dataset("json", data_files=src["data_files"], split=src["split"],
                                     streaming=True)
    return datasets.load_dataset(src["name"], src["config"], split=src["split"], streaming=True)


def prepare_source_stream(dataset, src, packer, seed: int, dp_rank: int, dp_size: int):
    from datasets.distributed import split_dataset_by_node

    if src["text_field"] != "text":
        dataset = dataset.rename_column(src["text_field"], "text")
    columns = dataset.column_names or list(next(iter(dataset)))
    dataset = dataset.shuffle(buffer_size=src["shuffle_buffer"], seed=seed)
    dataset = split_dataset_by_node(dataset, rank=dp_rank, world_size=dp_size)
    return dataset.map(packer, batched=True, batch_size=src["pack_batch"], remove_columns=columns)


def build_source_stream(src, packer, seed, dp_rank, dp_size):
    ds = load_source(src)
    if dp_rank == 0:
        print(f"{src['label']}: {ds.num_shards} shards, {src['weight']:.1%} of tokens")
    return prepare_source_stream(ds, src, packer, seed, dp_rank, dp_size)


def mixing_seed(seed: int, dp_rank: int) -> int:
    return seed + 10_000 + dp_rank


def mix_streams(streams, probabilities, seed: int, stopping_strategy: str = "all_exhausted"):
    assert len(streams) == len(probabilities), (
        f"{len(streams)} streams but {len(probabilities)} probabilities"
    )
    assert stopping_strategy in STOPPING_STRATEGIES, f"unknown stopping_strategy {stopping_strategy!r}"
    if len(streams) == 1:
        return streams[0]
    assert abs(sum(probabilities) - 1.0) < 1e-6, f"probabilities must sum to 1, got {sum(probabilities)}"
    import datasets

    return datasets.interleave_datasets(streams, probabilities=probabilities, seed=seed,
                                        stopping_strategy=stopping_strategy)


def build_synthetic_loader(data_cfg: dict, vocab_size: int, dp_rank: int, pin: bool = True):
    from pluggy_b200.dataloader.synthetic import SyntheticBatches, SyntheticZipfRows

    syn = dict(data_cfg.get("synthetic") or {})
    src = SyntheticZipfRows(vocab_size=vocab_size, seq_len=data_cfg["seq_len"],
                            eos_id=syn.get("eos_id"), seed=data_cfg.get("seed", 0), dp_rank=dp_rank,
                            zipf_s=syn.get("s", 1.1), min_doc=syn.get("min_doc", 512),
                            max_doc=syn.get("max_doc", 4096), kind=syn.get("kind", "zipf"))
    return SyntheticBatches(src, data_cfg["micro_batch_size"], pin=pin)


def build_dataloader(data_cfg, tokenizer, ignore_id: int, dp_rank: int, dp_size: int):
    from torchdata.stateful_dataloader import StatefulDataLoader

    sources = resolve_sources(data_cfg)
    eos_id = tokenizer.token_to_id(data_cfg["eos_token"])
    pad_id = tokenizer.token_to_id(data_cfg["pad_token"])
    assert eos_id is not None, f"eos_token {data_cfg['eos_token']!r} not in tokenizer vocab"
    assert pad_id is not None, f"pad_token {data_cfg['pad_token']!r} not in tokenizer vocab"
    packer = ListPacker(tokenizer, data_cfg["seq_len"], eos_id, pad_id)
    seed = data_cfg["seed"]
    streams = [build_source_stream(s, packer, seed + i, dp_rank, dp_size)
               for i, s in enumerate(sources)]
    mixing = data_cfg.get("mixing", {})
    dataset = mix_streams(streams, [s["weight"] for s in sources], seed=mixing_seed(seed, dp_rank),
                          stopping_strategy=mixing.get("stopping_strategy", "all_exhausted"))
    nw = data_cfg["num_workers"]
    if dp_rank == 0 and getattr(dataset, "num_shards", nw) < nw:
        print(f"warning: {nw} dataloader workers but the stream has {dataset.num_shards} shard(s)")
    return StatefulDataLoader(dataset, batch_size=data_cfg["micro_batch_size"], num_workers=nw,
                              collate_fn=Collator(tokenizer, ignore_id),
                              persistent_workers=nw > 0, pin_memory=torch.cuda.is_available())
