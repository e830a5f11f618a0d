"""LLM clients for the synthetic-data pipeline.

Parity: reference ``pluggy/synth/llm.py:16-74`` (Anthropic SDK client) and
``pluggy/synth/grok.py:24-91`` (xAI chat completions over stdlib HTTPS with retry
and backoff). Both expose ``generate_text(prompt, system=None, max_tokens=...)``
and ``generate_json(prompt, schema, system=None, max_tokens=...)`` and return None
when a request finally fails, so one bad document never stops a run.

The network clients need network access and an API key (``ANTHROPIC_API_KEY`` /
``XAI_API_KEY``). :class:`ScriptedClient` answers from a user function with no
network, for tests and dry runs.
"""

from __future__ import annotations

import json
import os
import random
import time
import urllib.error
import urllib.request


def _parse_json(text: str | None):
    """The first JSON object in ``text`` (models sometimes wrap it in prose or fences)."""
    if text is None:
        return None
    s = text.strip()
    if s.startswith("```"):
        s = s.strip("`")
        s = s[s.find("\n") + 1:] if "\n" in s else s
    i, j = s.find("{"), s.rfind("}")
    if i < 0 or j <= i:
        return None
    try:
        return json.loads(s[i:j + 1])
    except json.JSONDecodeError:
        return None


def _schema_ok(obj, schema: dict) -> bool:
    """Minimal check of an object against a JSON-schema subset (type + required keys)."""
    if schema.get("type") == "object":
        if not isinstance(obj, dict):
            return False
        for k in schema.get("required", []):
            if k not in obj:
                return False
        for k, sub in schema.get("properties", {}).items():
            if k in obj and not _schema_ok(obj[k], sub):
                return False
        return True
    if schema.get("type") == "array":
        return isinstance(obj, list) and all(_schema_ok(x, schema.get("items", {})) for x in obj)
    if schema.get("type") == "string":
        return isinstance(obj, str)
    if schema.get("type") in ("integer", "number"):
        return isinstance(obj, (int, float)) and not isinstance(obj, bool)
    return True


class _Base:
    def generate_text(self, prompt: str, system: str | None = None, max_tokens: int = 4096):
        raise NotImplementedError

    def generate_json(self, prompt: str, schema: dict, system: str | None = None,
                      max_tokens: int = 2048):
        guide = ("Reply with one JSON object and nothing else, matching this JSON schema:\n"
                 + json.dumps(schema))
        text = self.generate_text(prompt + "\n\n" + guide, system=system, max_tokens=max_tokens)
        obj = _parse_json(text)
        return obj if obj is not None and _schema_ok(obj, schema) else None


class GrokClient(_Base):
    """xAI chat completions over HTTPS (stdlib only), retrying transient failures."""

    API_URL = "https://api.x.ai/v1/chat/completions"
    RETRYABLE = {408, 409, 429, 500, 502, 503, 504, 529}

    def __init__(self, model: str, temperature: float | None = None, max_retries: int = 5,
                 timeout_s: float = 600.0):
        self.model, self.temperature = model, temperature
        self.max_retries, self.timeout_s = max_retries, timeout_s
        self.key = os.environ.get("XAI_API_KEY")

    def _post(self, payload: dict) -> dict | None:
        if not self.key:
            raise RuntimeError("XAI_API_KEY is not set")
        body = json.dumps(payload).encode()
        for attempt in range(self.max_retries + 1):
            req = urllib.request.Request(self.API_URL, data=body, method="POST", headers={
                "Authorization": f"Bearer {self.key}", "Content-Type": "application/json"})
            try:
                with urllib.request.urlopen(req, timeout=self.timeout_s) as r:
                    return json.loads(r.read())
            except urllib.error.HTTPError as e:
                if e.code not in self.RETRYABLE or attempt == self.max_retries:
                    return None
            except (urllib.error.URLError, TimeoutError):
                if attempt == self.max_retries:
                    return None
            time.sleep(min(60.0, 2.0 ** attempt) * (0.5 + random.random()))
        return None

    def generate_text(self, prompt, system=None, max_tokens=4096):
        msgs = ([{"role": "system", "content": system}] if system else []) + [
            {"role": "user", "content": prompt}]
        payload = {"model": self.model, "messages": msgs, "max_tokens": max_tokens}
        if self.temperature is not None:
            payload["temperature"] = self.temperature
        out = self._post(payload)
        try:
            return out["choices"][0]["message"]["content"] if out else None
        except (KeyError, IndexError, TypeError):
            return None


class AnthropicClient(_Base):
    """Claude models through the ``anthropic`` SDK (imported on first use)."""

    def __init__(self, model: str, max_retries: int = 5):
        self.model, self.max_retries = model, max_retries
        self._sdk = None

    def _client(self):
        if self._sdk is None:
            import anthropic  # noqa: PLC0415 - optional dependency

            self._sdk = anthropic.Anthropic(max_retries=self.max_retries)
        return self._sdk

    def generate_text(self, prompt, system=None, max_tokens=4096):
        kw = {"model": self.model, "max_tokens": max_tokens,
              "messages": [{"role": "user", "content": prompt}]}
        if system:
            kw["system"] = system
        try:
            r = self._client().messages.create(**kw)
        except Exception:  # noqa: BLE001 - a failed document is dropped, not fatal
            return None
        parts = [getattr(b, "text", "") for b in getattr(r, "content", [])]
        return "".join(parts) or None


class ScriptedClient(_Base):
    """Answers with ``fn(prompt, system, max_tokens) -> str`` (no network)."""

    def __init__(self, fn):
        self.fn = fn
        self.calls = 0

    def generate_text(self, prompt, system=None, max_tokens=4096):
        self.calls += 1
        return self.fn(prompt, system, max_tokens)


def build_client(cfg: dict):
    """``cfg["provider"]`` ("grok" / "anthropic"), else inferred from the model name."""
    model = cfg.get("model", "grok-4")
    provider = cfg.get("provider") or ("grok" if model.startswith("grok") else "anthropic")
    if provider == "grok":
        return GrokClient(model, temperature=cfg.get("generation", {}).get("temperature"))
    if provider == "anthropic":
        return AnthropicClient(model)
    raise ValueError(f"unknown provider {provider!r}: expected 'grok' or 'anthropic'")
