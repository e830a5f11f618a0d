"""``python -m pluggy_b200.synth.run --config synth.json``: run the synthetic-data pipeline.

Parity: reference ``pluggy/synth/run.py``. Credentials follow the provider:
``XAI_API_KEY`` for grok (stdlib HTTPS), ``ANTHROPIC_API_KEY`` and the ``anthropic``
package for Claude models.
"""

from __future__ import annotations

import argparse
import json

from pluggy_b200.synth.pipeline import run_pipeline


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", required=True)
    a = p.parse_args(argv)
    with open(a.config) as f:
        run_pipeline(json.load(f))


if __name__ == "__main__":
    main()
