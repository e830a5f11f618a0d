"""Synthetic pretraining data: an LLM generate -> judge -> refine loop over a topic
taxonomy and/or uploaded source text, deduplicated into JSONL shards whose ``text``
column feeds the framework's data loader directly."""
