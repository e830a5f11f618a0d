"""Grounded synthesis: documents written from chunks of user-supplied text.

Parity: reference ``pluggy/synth/grounded.py:18-83``: the four modes, and
deterministic word-window chunking of every ``*.jsonl`` (rows with ``"text"``) in a
directory, dropping tails shorter than a quarter window; the chunk index is the
job key, so the chunking must not change under a resume.
"""

from __future__ import annotations

import json
from pathlib import Path

GROUNDED_MODES = {
    "rephrase": "the source restated as clean, well-organised expository prose that keeps "
                "every fact, figure and caveat",
    "textbook": "a textbook section that supplies the background a newcomer lacks, defines "
                "terms and builds up to the source's specifics",
    "qa": "a question-and-answer dialogue several rounds deep through the source's content, "
          "asking what a real reader would ask",
    "summary": "a dense summary of the source followed by an analysis of what it implies "
               "and how its parts connect",
}

SYSTEM = ("You write language-model pretraining documents from a source text. Every specific "
          "claim (figures, names, procedures, interfaces) must come from the source; general "
          "background knowledge is allowed, invented specifics are not. Output only the "
          "document, without remarks about the source or the task.")

PROMPT = ("<source>\n{chunk}\n</source>\n\nForm: {mode}\n\nThis is document {variant} of "
          "several written from this source: take an angle other than the obvious one.")


def load_chunks(src_dir, chunk_words: int) -> list[str]:
    files = sorted(Path(src_dir).glob("*.jsonl"))
    if not files:
        raise FileNotFoundError(f"no *.jsonl files in {src_dir}: upload data first, or put "
                                "normalised {\"text\": ...} rows there")
    min_words = max(1, chunk_words // 4)
    out = []
    for fp in files:
        with open(fp, encoding="utf-8") as f:
            for line in f:
                if not line.strip():
                    continue
                words = json.loads(line)["text"].split()
                for i in range(0, len(words), chunk_words):
                    piece = words[i:i + chunk_words]
                    if len(piece) >= min_words:
                        out.append(" ".join(piece))
    return out


def generate_grounded(client, chunk: str, mode: str, variant: int, max_tokens: int):
    text = client.generate_text(
        PROMPT.format(chunk=chunk, mode=GROUNDED_MODES[mode], variant=variant + 1),
        system=SYSTEM, max_tokens=max_tokens)
    if text is None or len(text.strip()) < 200:
        return None
    return text.strip()
