"""Reference arm of ``bench.py``: the unmodified ``nano_vllm_uno`` package.

Installed offline into ``baseline/_ref``; not wired up yet.
"""

import json


def run(args):
    print(json.dumps({"impl": "reference", "unavailable": "reference arm not wired up yet"}), flush=True)
