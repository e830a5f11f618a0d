"""Topic documents: a (topic, style, variant) grid.

Parity: reference ``pluggy/synth/generate.py:9-46``.
"""

from __future__ import annotations

STYLES = {
    "textbook": "a textbook section that defines its terms and develops the ideas in order",
    "tutorial": "a practical tutorial that works through concrete, runnable examples",
    "qa": "a multi-turn dialogue in which a learner questions an expert in depth",
    "essay": "an argumentative essay that takes a position and answers objections",
    "reference": "terse, exhaustive reference documentation for a narrow scope",
}

SYSTEM = ("You write documents for a language-model pretraining corpus: accurate, dense, "
          "written the way a careful expert writes. Output only the document, with no "
          "preamble, no commentary about the task and no placeholders.")

PROMPT = ("Domain: {domain}\nTopic: {topic} ({summary})\nForm: {style}\n\n"
          "This is variant {variant}: choose an angle, emphasis or entry point that the "
          "other variants are unlikely to take, while staying substantive.")


def generate_doc(client, topic: dict, style: str, variant: int, max_tokens: int) -> str | None:
    text = client.generate_text(
        PROMPT.format(domain=topic["domain"], topic=topic["topic"],
                      summary=topic.get("summary", ""), style=STYLES[style], variant=variant),
        system=SYSTEM, max_tokens=max_tokens)
    if text is None or len(text.strip()) < 200:
        return None
    return text.strip()
