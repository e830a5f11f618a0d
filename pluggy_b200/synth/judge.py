"""Quality gate: judge -> (refine -> re-judge) for one document.

Parity: reference ``pluggy/synth/judge.py:78-119``. A judge call scores the
document 1..10 with a short list of weaknesses; a score >= ``min_score`` keeps it,
a score in ``[refine_min, min_score)`` earns up to ``max_refine_rounds`` rewrites
that are fed the weaknesses, anything lower (or any failed call) drops it. A
grounded document is judged against its source, with faithfulness first.
"""

from __future__ import annotations

SCHEMA = {
    "type": "object",
    "required": ["score", "weaknesses"],
    "properties": {"score": {"type": "integer"}, "weaknesses": {"type": "string"}},
}

RUBRIC = (
    "Rate the document below as language-model pretraining data with one integer from 1 "
    "to 10. Factual errors or internal contradictions cap the score at 4. Reward how much "
    "it teaches per token, depth beyond a surface summary, and clear expert prose; "
    "penalise filler and repetition. 8-10 strong, 5-7 usable with flaws, 1-4 reject. "
    "Name the main weaknesses in one or two sentences.\n\n<document>\n{doc}\n</document>"
)

RUBRIC_GROUNDED = (
    "Rate the document below as language-model pretraining data with one integer from 1 "
    "to 10. It was written from the source that follows. First criterion: every specific "
    "(figure, name, procedure) must be supported by the source; invented specifics cap the "
    "score at 4. Then: how well it uses the source's substance, and clear expert prose. "
    "Name the main weaknesses in one or two sentences.\n\n<source>\n{source}\n</source>\n\n"
    "<document>\n{doc}\n</document>"
)

REWRITE = (
    "Rewrite this document so that these weaknesses are gone, keeping its subject, form "
    "and angle. Output only the new document.\n\nWeaknesses: {weak}\n\n<document>\n{doc}\n"
    "</document>"
)


def judge_doc(client, doc: str, source: str | None = None) -> dict | None:
    prompt = (RUBRIC.format(doc=doc) if source is None
              else RUBRIC_GROUNDED.format(doc=doc, source=source))
    v = client.generate_json(prompt, SCHEMA, max_tokens=1024)
    if v is None or not isinstance(v.get("score"), int) or not 1 <= v["score"] <= 10:
        return None
    return v


def refine_doc(client, doc: str, weaknesses: str, max_tokens: int) -> str | None:
    text = client.generate_text(REWRITE.format(weak=weaknesses, doc=doc), max_tokens=max_tokens)
    if text is None or len(text.strip()) < 200:
        return None
    return text.strip()


def evaluate(client, doc: str, quality_cfg: dict, max_tokens: int, source: str | None = None):
    """``(doc, score)`` of the kept (possibly rewritten) document, or ``(None, None)``."""
    keep_at = quality_cfg.get("min_score", 7)
    refine_at = quality_cfg.get("refine_min", 5)
    rounds = quality_cfg.get("max_refine_rounds", 1)
    v = judge_doc(client, doc, source)
    r = 0
    while v is not None and v["score"] < keep_at:
        if v["score"] < refine_at or r >= rounds:
            return None, None
        doc = refine_doc(client, doc, v["weaknesses"], max_tokens)
        if doc is None:
            return None, None
        v = judge_doc(client, doc, source)
        r += 1
    if v is None:
        return None, None
    return doc, v["score"]
