"""pck — the checked decode path of proof-carrying-kernels, rebuilt for B200 (sm_100a).

`pck.cuda` holds the GPU API (GEMVs, the trusted blocked checker, the sampling checks);
`pck.member.check_members` is the fused sampled-token membership check; `pck.fp` the
host-side rounding constants. Every GPU entry point runs a kernel of libpck_b200.so.
"""

from pck.fp import U32, U64, bf16, ceil_div, gamma, next_up, softmax_eps, sum_up_factor, tree_height

__all__ = [
    "U32",
    "U64",
    "bf16",
    "ceil_div",
    "gamma",
    "next_up",
    "softmax_eps",
    "sum_up_factor",
    "tree_height",
]
