"""The hash-pinned trusted sources (pck.manifest, the drop-in for src/pck/manifest.py): the
pin is current, a changed trusted file is named until it is re-pinned, the loaded library
was built from the sources on disk, and run certificates round-trip. CPU only."""

from __future__ import annotations

import json
import shutil
from pathlib import Path

import pytest

from pck import manifest


def _copy_trusted(dst: Path) -> None:
    for rel in manifest.TRUSTED:
        (dst / rel).parent.mkdir(parents=True, exist_ok=True)
        shutil.copy2(manifest.ROOT / rel, dst / rel)
    # the build's digest reads every library source, not only the trusted ones
    pkg = manifest.ROOT / "proof-carrying-kernels_b200"
    for sub in ("csrc",):
        for f in (pkg / sub).iterdir():
            shutil.copy2(f, dst / "proof-carrying-kernels_b200" / sub / f.name)
    (dst / "include").mkdir(exist_ok=True)
    for f in (manifest.ROOT / "include").glob("*.h"):
        shutil.copy2(f, dst / "include" / f.name)


def test_the_pin_is_current_and_the_library_matches_its_sources() -> None:
    manifest.verify_pinned(library=False)
    assert manifest.checker_hash() == manifest.pinned()["checker"]
    assert set(manifest.pinned()["files"]) == set(manifest.TRUSTED)
    assert manifest.library_digest() == manifest.source_digest()


def test_a_changed_trusted_file_is_named_until_repinned(tmp_path: Path) -> None:
    _copy_trusted(tmp_path)
    lock = tmp_path / "lock.json"
    shutil.copy2(manifest.LOCK, lock)
    manifest.verify_pinned(root=tmp_path, lock=lock, library=False)
    target = tmp_path / "proof-carrying-kernels_b200/csrc/verdict_kernel.cu"
    target.write_bytes(target.read_bytes() + b"\n// a reviewed change\n")
    with pytest.raises(manifest.CheckerMismatch, match="verdict_kernel.cu"):
        manifest.verify_pinned(root=tmp_path, lock=lock, library=False)
    # the library built from the original sources no longer matches them
    assert manifest.source_digest(tmp_path) != manifest.source_digest()
    pinned = manifest.update(root=tmp_path, lock=lock)
    assert json.loads(lock.read_text())["checker"] == pinned
    manifest.verify_pinned(root=tmp_path, lock=lock, library=False)


def test_a_manifest_round_trips_and_reports_a_stale_pin(tmp_path: Path) -> None:
    cert = manifest.Manifest(workload="test", config={"batch": 1}, measured={"passed": True},
                             library=manifest.library_digest())  # fmt: skip
    again = manifest.Manifest.from_json(cert.to_json())
    assert again == cert
    assert cert.problems() == []
    assert set(cert.theorems) == set(manifest.THEOREMS) and cert.hypotheses
    stale = tmp_path / "lock.json"
    stale.write_text(json.dumps({"checker": "0" * 64, "files": {}}))
    assert "checker hash differs from the pinned checker" in cert.problems(lock=stale)
