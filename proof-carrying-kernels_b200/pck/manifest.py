"""Hash-pinned trusted sources of the checked decode path, and run certificates.

What a verdict of this library rests on is a short list of files: the kernels that compute
the checksum-bank sums and decide the blocks, the membership and set checkers, the launch
planning and argument checks around them, the host-side constants of the proven bound, the
compiler flags, and the plugin that feeds vLLM's sampled tokens to the membership check.
Their SHA-256 hashes are pinned in ``trusted_lock.json`` (the drop-in for the reference's
checker_lock.json, src/pck/manifest.py:27-98). `verify_pinned` refuses to vouch for a run if
a trusted file on disk differs from its pin, or if the loaded libpck_b200.so was not built
from the sources on disk (its compiled-in `pck_source_digest()` against the build's digest
of them). A `Manifest` records, for one checked run, the pin it ran under, the library's
digest, the theorems the bound rests on, the commit and the measured figures.

Re-pin after a reviewed change to a trusted file:
    python -m pck.manifest --update
"""

from __future__ import annotations

import argparse
import functools
import hashlib
import importlib.util
import json
import subprocess
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

PACKAGE = Path(__file__).resolve().parent  # pck/
ROOT = PACKAGE.parents[1]  # the repository (trusted paths are relative to it)
LOCK = PACKAGE / "trusted_lock.json"

TRUSTED = (
    # device code whose arithmetic the verdicts rest on
    "proof-carrying-kernels_b200/csrc/verdict_kernel.cu",  # the decision rule
    "proof-carrying-kernels_b200/csrc/verdict_task.cuh",
    "proof-carrying-kernels_b200/csrc/verdict_plan.h",  # segment split the verdicts read
    "proof-carrying-kernels_b200/csrc/stream_kernel.cuh",  # bank units of the batch-1 path
    "proof-carrying-kernels_b200/csrc/tc_kernel.cu",  # bank warps of the tensor-core path
    "proof-carrying-kernels_b200/csrc/bank_batch_kernel.cu",
    "proof-carrying-kernels_b200/csrc/bank_kernel.cu",  # c and a at weight load
    "proof-carrying-kernels_b200/csrc/member_kernel.cu",
    "proof-carrying-kernels_b200/csrc/sampling_kernel.cu",
    "proof-carrying-kernels_b200/csrc/pck_common.cuh",  # bounded waits, conversions
    "proof-carrying-kernels_b200/csrc/capi.cu",  # argument checks, plans, which checks run
    "proof-carrying-kernels_b200/csrc/static_scratch.cu",
    "include/pck_b200.h",
    "proof-carrying-kernels_b200/build.py",  # --fmad=false, IEEE division, no flush to zero
    # host code that computes the bound's constants and builds the checks' inputs
    "proof-carrying-kernels_b200/pck/fp.py",
    "proof-carrying-kernels_b200/pck/cuda/checker.py",
    "proof-carrying-kernels_b200/pck/cuda/gemv.py",  # tc_height, the declared tensor-core height
    "proof-carrying-kernels_b200/pck/cuda/sampling.py",
    "proof-carrying-kernels_b200/pck/member.py",
    "proof-carrying-kernels_b200/pck/vllm_plugin.py",
)

THEOREMS = {
    "T1 no false alarms": "PCK.t1_block",
    "T2 guaranteed detection": "PCK.t2_block",
    "T3 safe runtime threshold": "PCK.t3_no_false_alarm",
    "T4 randomized detection": "PCK.t4_computed",
    "T4 spread errors": "PCK.t4_spread_computed",
}
"""The Lean theorems of the reference project the checker's bound and verdicts rest on."""

TC_HYPOTHESIS = ("each tcgen05.mma step is within 8 unit roundoffs of |accumulator| + sum |products| "
                 "(pck.cuda.gemv.tc_height); tested, not proven")  # fmt: skip
"""The assumption behind checks of the tensor-core GEMV, recorded in every manifest."""


class CheckerMismatch(RuntimeError):
    """The trusted sources on disk, or the loaded library, are not the pinned ones."""


@functools.lru_cache(maxsize=256)
def _digest(path: str, mtime_ns: int, size: int) -> str:
    del mtime_ns, size  # cache keys: a changed file is hashed again
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def file_hash(rel: str, root: Path = ROOT) -> str:
    """SHA-256 of a trusted file (re-read only when its size or modification time changes)."""
    path = root / rel
    st = path.stat()
    return _digest(str(path), st.st_mtime_ns, st.st_size)


def file_hashes(root: Path = ROOT) -> dict[str, str]:
    return {rel: file_hash(rel, root) for rel in TRUSTED}


def combined(hashes: dict[str, str]) -> str:
    """One hash over (path, file hash) pairs in path order."""
    h = hashlib.sha256()
    for rel in sorted(hashes):
        h.update(f"{rel}\t{hashes[rel]}\n".encode())
    return h.hexdigest()


def checker_hash(root: Path = ROOT) -> str:
    return combined(file_hashes(root))


def pinned(lock: Path = LOCK) -> dict[str, Any]:
    data: dict[str, Any] = json.loads(lock.read_text())
    return data


def _build_module(root: Path = ROOT):
    spec = importlib.util.spec_from_file_location("_pck_build", root / "proof-carrying-kernels_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def source_digest(root: Path = ROOT) -> str:
    """The build's digest of the library sources on disk (what pck_source_digest() of a
    library built from them returns)."""
    return _build_module(root).source_digest()


def library_digest() -> str:
    """The digest compiled into the loaded libpck_b200.so."""
    from pck.cuda import _lib

    return _lib.library().pck_source_digest().decode()


def verify_pinned(root: Path = ROOT, lock: Path = LOCK, library: bool = True) -> None:
    """Raise `CheckerMismatch` naming what differs: trusted files whose hash is not the pinned
    one, and (``library``) a loaded library built from other sources than those on disk."""
    pin = pinned(lock)
    now = file_hashes(root)
    problems = []
    if combined(now) != pin.get("checker"):
        changed = sorted(rel for rel in TRUSTED if pin.get("files", {}).get(rel) != now[rel])
        stale = sorted(set(pin.get("files", {})) - set(TRUSTED))
        problems.append("trusted sources differ from the pin (" + ", ".join(changed + stale) + ")")
    if library and library_digest() != source_digest(root):
        problems.append("the loaded libpck_b200.so was built from other sources than those on disk; rebuild it")
    if problems:
        raise CheckerMismatch("; ".join(problems) + "; review the change, then run: python -m pck.manifest --update")


def update(root: Path = ROOT, lock: Path = LOCK) -> str:
    """Pin the trusted files as they are now; returns the combined hash."""
    hashes = file_hashes(root)
    lock.write_text(json.dumps({"checker": combined(hashes), "files": hashes}, indent=2, sort_keys=True) + "\n")
    return combined(hashes)


@functools.cache
def git_commit(root: Path = ROOT) -> str | None:
    """HEAD of the checkout, once per process."""
    try:
        out = subprocess.run(["git", "rev-parse", "HEAD"], cwd=root, capture_output=True, text=True, check=True)
    except (OSError, subprocess.CalledProcessError):
        return None
    return out.stdout.strip() or None


@dataclass(frozen=True)
class Manifest:
    """The certificate of one checked run: what ran (workload, config), what it was checked
    with (pinned checker hash, library digest, the theorems and the tensor-core hypothesis)
    and what was measured."""

    workload: str
    config: dict[str, Any]
    measured: dict[str, Any]
    checker: str = field(default_factory=checker_hash)
    library: str | None = None
    theorems: dict[str, str] = field(default_factory=lambda: dict(THEOREMS))
    hypotheses: tuple[str, ...] = (TC_HYPOTHESIS,)
    commit: str | None = field(default_factory=git_commit)

    def to_json(self) -> str:
        return json.dumps(asdict(self), indent=2, sort_keys=True) + "\n"

    @classmethod
    def from_json(cls, text: str) -> Manifest:
        data = json.loads(text)
        data["hypotheses"] = tuple(data.get("hypotheses", ()))
        return cls(**data)

    def problems(self, lock: Path = LOCK) -> list[str]:
        """Why this certificate does not match the pinned checker (empty: it does)."""
        out = []
        if self.checker != pinned(lock)["checker"]:
            out.append("checker hash differs from the pinned checker")
        if self.library is not None and self.library != source_digest():
            out.append("library digest differs from the sources on disk")
        return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--update", action="store_true", help="re-pin the trusted files as they are now")
    parser.add_argument("--no-library", action="store_true", help="skip the loaded-library check")
    args = parser.parse_args()
    if args.update:
        print(f"pinned {update()}")
        return
    try:
        verify_pinned(library=not args.no_library)
        print(f"trusted sources match the pin {checker_hash()}")
    except CheckerMismatch as e:
        print(e)
        raise SystemExit(1) from None


if __name__ == "__main__":
    main()
