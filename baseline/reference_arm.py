"""Reference arm of bench.py: runs the reference's own Wan DMAD code from baseline/_ref.

The reference repository has no setup.py / pyproject.toml, so `pip install` of it fails
("Neither 'setup.py' nor 'pyproject.toml' found"); see DESIGN.md.  Until an installed copy
exists under baseline/_ref this arm prints its `unavailable` line.
"""
from __future__ import annotations

import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def build_reference_trainer(args, device):
    if not os.path.isdir(os.path.join(REF, "rcm")):
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference has no setup.py/pyproject.toml; pip install into baseline/_ref failed"}))
        return None
    raise NotImplementedError
