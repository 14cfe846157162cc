"""The reference arm's self-install: with baseline/_ref missing and a reference checkout present, the Wan
trees are pip-installed (offline, no dependencies) beside a copy of the image stack; with neither, it
reports that it cannot."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _fake_checkout(base):
    for d in ("train/wan/rcm/networks", "train/wan/imaginaire/utils", "train/image/main", "train/image/third_party/edm"):
        os.makedirs(os.path.join(base, d), exist_ok=True)
    for f in ("train/wan/rcm/__init__.py", "train/wan/rcm/networks/__init__.py", "train/wan/imaginaire/__init__.py",
              "train/wan/imaginaire/utils/__init__.py"):
        with open(os.path.join(base, f), "w") as fh:
            fh.write("")
    with open(os.path.join(base, "train/wan/rcm/networks/wan2pt1.py"), "w") as fh:
        fh.write("MARKER = 1\n")
    with open(os.path.join(base, "train/image/main/utils.py"), "w") as fh:
        fh.write("")


def test_provision_installs_from_checkout(tmp_path, monkeypatch):
    sys.path.insert(0, ROOT)
    from baseline import reference_arm as arm

    ck, ref = str(tmp_path / "ref_checkout"), str(tmp_path / "_ref")
    _fake_checkout(ck)
    monkeypatch.setattr(arm, "REF", ref)
    monkeypatch.setattr(arm, "_reference_checkout", lambda: ck)
    assert arm.provision(log=open(os.devnull, "w"))
    assert os.path.isfile(os.path.join(ref, "rcm", "networks", "wan2pt1.py"))
    assert os.path.isdir(os.path.join(ref, "imaginaire", "utils"))
    assert os.path.isfile(os.path.join(ref, "image", "main", "utils.py"))
    assert os.path.isdir(os.path.join(ref, "image", "third_party", "edm"))
    assert arm.provision()  # already in place: nothing to do


def test_provision_without_checkout_reports_missing(tmp_path, monkeypatch):
    sys.path.insert(0, ROOT)
    from baseline import reference_arm as arm

    monkeypatch.setattr(arm, "REF", str(tmp_path / "_ref"))
    monkeypatch.setattr(arm, "_reference_checkout", lambda: None)
    assert not arm.provision()
