"""Topic taxonomy: one structured LLM call per seed domain.

Parity: reference ``pluggy/synth/taxonomy.py:32-45``: each domain expands into
``subtopics_per_domain`` topics; every topic gets a stable id so resumed runs map
work to the same keys.
"""

from __future__ import annotations

SCHEMA = {
    "type": "object",
    "required": ["topics"],
    "properties": {"topics": {"type": "array", "items": {
        "type": "object", "required": ["topic", "summary"],
        "properties": {"topic": {"type": "string"}, "summary": {"type": "string"}}}}},
}

PROMPT = (
    "Break the field \"{domain}\" into {n} distinct, substantive subtopics that together "
    "cover it for a reader building expert-level understanding. Give each a short title "
    "(\"topic\") and a one-sentence scope (\"summary\"). Avoid overlap between subtopics."
)


def build_taxonomy(client, domains: list[str], subtopics_per_domain: int) -> list[dict]:
    out = []
    for di, domain in enumerate(domains):
        res = client.generate_json(PROMPT.format(domain=domain, n=subtopics_per_domain), SCHEMA)
        if res is None:
            raise RuntimeError(f"taxonomy call failed for domain {domain!r}")
        for ti, t in enumerate(res["topics"][:subtopics_per_domain]):
            out.append({"id": f"d{di}t{ti}", "domain": domain, "topic": t["topic"],
                        "summary": t["summary"]})
    return out
