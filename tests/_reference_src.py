"""Where the reference's source lives for the CPU oracles.

Order: the offline install under ``baseline/_ref`` (the Wan trees ``rcm`` / ``imaginaire``), else the
reference checkout named by ``reference_path`` in the repository's ``BASELINE.json``.  When neither is
present the oracle tests fail: they are the evidence that the models match the reference, and a
silent skip would hide their absence."""
import json
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INSTALLED = os.path.join(ROOT, "baseline", "_ref")


def _checkout():
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            path = json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None
    return path if path and os.path.isdir(path) else None


def wan_tree() -> str:
    """Directory holding the reference's ``rcm`` and ``imaginaire`` packages."""
    if os.path.isdir(os.path.join(INSTALLED, "rcm")):
        return INSTALLED
    ck = _checkout()
    if ck and os.path.isdir(os.path.join(ck, "train", "wan", "rcm")):
        return os.path.join(ck, "train", "wan")
    pytest.fail("the reference source is neither installed under baseline/_ref nor checked out at BASELINE.json's "
                "reference_path: the oracle cannot run")


def image_tree() -> str:
    """The reference's image stack (``main/`` and ``third_party/edm``)."""
    for base in (os.path.join(INSTALLED, "image"), os.path.join(_checkout() or "", "train", "image")):
        if os.path.isdir(os.path.join(base, "third_party", "edm")):
            return base
    pytest.fail("the reference image stack is neither under baseline/_ref/image nor in the reference checkout")
