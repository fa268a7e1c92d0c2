"""CPU oracle for the checked decode path — TEST INFRASTRUCTURE ONLY.

Nothing in the product (`pck`, the CUDA library) imports, links or runs this package.
Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline legs of `bench.py` use it,
and there only as the checker of the GPU results or as the timed CPU reference.

Each module restates, in code written for this repository, an algorithm of the
reference project r7919/proof-carrying-kernels (cited as ``file:line`` relative to that
project's root):

- `oracle.fp`       — rounding helpers and error constants   (src/pck/fp.py)
- `oracle.gemv`     — bit-faithful GEMV summation-tree models  (src/pck/gemv.py)
- `oracle.checker`  — CPU blocked checker, and the GPU checker's bank and verdict
                      arithmetic                                (src/pck/checker.py,
                      src/pck/cuda/checker.py, src/pck/cuda/csrc/checker_kernel.cu)
- `oracle.member`   — sampled-token membership check           (src/pck/member.py)
- `oracle.sampling` — top-k / top-p set checks and samplers     (src/pck/sampling.py)
- `oracle.faults`   — fault models                              (src/pck/faults.py)
- `oracle/gemv_ref.c` — the coalesced GEMV model in C (OpenMP over rows), for
                      full-size parity and the timed CPU baseline.

Parity is pinned: `tests/golden/make_golden.py` ran the reference's own Python code in the
build container and froze its outputs under `tests/golden/`; `tests/test_oracle_golden.py`
checks every function here against those fixtures.
"""
