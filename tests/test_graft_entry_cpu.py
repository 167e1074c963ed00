"""build()'s helper that recreates the verbatim copy of the reference used by
bench.py's reference arm (the reference ships no packaging metadata, so the
copy stands in for an install): it copies the checkout BASELINE.json names
when the copy is missing and leaves an existing copy alone."""
import json
import os

import __graft_entry__ as entry


def _fake_tree(tmp_path):
    ref = tmp_path / "reference"
    ref.mkdir()
    (ref / "slide_fsdp.py").write_text("# stand-in\n")
    (ref / "config.py").write_text("X = 1\n")
    root = tmp_path / "repo"
    (root / "baseline").mkdir(parents=True)
    (root / "BASELINE.json").write_text(json.dumps({"reference_path": str(ref)}))
    return root, ref


def test_reference_copy_made_when_missing(tmp_path, monkeypatch):
    root, ref = _fake_tree(tmp_path)
    monkeypatch.setattr(entry, "ROOT", str(root))
    entry._materialize_reference()
    dst = root / "baseline" / "_ref"
    assert (dst / "slide_fsdp.py").read_text() == "# stand-in\n"
    assert (dst / "config.py").exists()


def test_existing_reference_copy_left_alone(tmp_path, monkeypatch):
    root, ref = _fake_tree(tmp_path)
    dst = root / "baseline" / "_ref"
    dst.mkdir()
    (dst / "slide_fsdp.py").write_text("# already here\n")
    monkeypatch.setattr(entry, "ROOT", str(root))
    entry._materialize_reference()
    assert (dst / "slide_fsdp.py").read_text() == "# already here\n"
    assert not (dst / "config.py").exists()


def test_missing_reference_checkout_is_not_an_error(tmp_path, monkeypatch):
    root = tmp_path / "repo"
    (root / "baseline").mkdir(parents=True)
    (root / "BASELINE.json").write_text(json.dumps({"reference_path": str(tmp_path / "nowhere")}))
    monkeypatch.setattr(entry, "ROOT", str(root))
    entry._materialize_reference()
    assert not os.path.exists(root / "baseline" / "_ref")
