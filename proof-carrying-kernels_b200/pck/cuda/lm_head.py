"""Row-sharded, checked LM head with top-k / top-p sampling and the sampled-token membership
check: one decode step of the output layer, on one GPU or row-sharded over the GPUs of a node.

The vocabulary rows of W (V, n) are split by whole checker blocks (`shard_rows`); each rank
runs the tensor-core GEMV of its slice for the decode batch X (B, n) with the slice's blocked
check fused into the same call (`pck_gemv_tc`, checker height `tc_height(n)`), writing its
logits and verdict bits into one packed buffer. One all-gather per step assembles every
rank's logits and verdicts (NCCL over NVLink); every rank then holds the full (B, V) logits,
samples from them and checks the sampled tokens with the fused membership kernel
(`pck_member_check`, one launch for the batch), as the reference checks every sampled token
(src/pck/member.py:118-197, src/pck/vllm_plugin.py:132-197).

The sampler is untrusted torch code (the vLLM sampler's semantics: temperature, the k
largest logits, then the shortest prefix of them whose probability reaches p, then one
draw); the tokens it returns are what the membership check certifies. Fault injection
replaces a share of the sampled tokens with the row's lowest logit, which no correct top-k /
top-p sampler returns (the reference plugin's PCK_FAULT_RATE model, src/pck/vllm_plugin.py:174-182).
Every step draws its random numbers from torch's default CUDA generator into fixed buffers,
so a step can be captured in a CUDA graph and replayed.
"""

from __future__ import annotations

import torch

from pck.cuda.checker import GpuBlockedChecker
from pck.cuda.gemv import tc_height
from pck.cuda.plan import TcLaunch
from pck.cuda.sharded import Exchange, shard_rows
from pck.member import check_members


class CheckedLMHead:
    """The LM head of one rank: the rows of its shard of W, their checker, and the packed
    exchange of logits and verdict bits.

    ``W_local`` is this rank's slice (rows ``shard_rows(vocab, block, world, rank)``) in
    bfloat16; ``X`` the decode batch (B, n) bfloat16, read at every `forward` (update it in
    place between steps). ``generator`` draws the checker's secret signs (CPU generator, as
    GpuBlockedChecker).
    """

    def __init__(self, W_local: torch.Tensor, X: torch.Tensor, vocab: int, block: int = 128, checks: int = 1,
                 world: int = 1, rank: int = 0, generator: torch.Generator | None = None) -> None:  # fmt: skip
        shard = shard_rows(vocab, block, world, rank)
        if W_local.dtype != torch.bfloat16 or W_local.dim() != 2 or W_local.size(0) != shard.rows:
            raise ValueError(f"W_local must be the bfloat16 rows [{shard.row0}, {shard.row1}) of W")
        if X.dtype != torch.bfloat16 or X.dim() != 2 or X.size(1) != W_local.size(1):
            raise ValueError("X must be a bfloat16 (B, n) batch with n = W's columns")
        self.vocab, self.block, self.checks, self.world, self.rank = vocab, block, checks, world, rank
        self.batch, self.n = X.size(0), X.size(1)
        self.device = W_local.device
        self.shard = shard
        self.X = X
        self.W = W_local
        self.checker = GpuBlockedChecker(W_local, block, tc_height(self.n), checks=checks, generator=generator)
        nb = vocab // block
        self.exchange = Exchange([([vocab], block, self.batch, torch.float32),
                                  ([nb], 1, self.batch * checks, torch.bool)], world, rank, self.device)  # fmt: skip
        logits_part, verdict_part = self.exchange.parts
        self.local_logits = logits_part.local_view(0)  # (B, rows of this shard)
        self.local_passed = verdict_part.local_view(0)  # (B * checks, blocks of this shard)
        self.gemv = TcLaunch([(W_local, X, self.checker)], ys=[self.local_logits], passed=[self.local_passed],
                             full_k=True)  # every rank's slice rounds as in the unsharded GEMV
        if world == 1:
            self.logits = self.local_logits  # (B, V)
            self.passed = self.local_passed.view(self.batch, checks, nb)
        else:
            self.logits = torch.empty((self.batch, vocab), dtype=torch.float32, device=self.device)
            self.passed = torch.empty((self.batch, checks, nb), dtype=torch.bool, device=self.device)

    def forward(self) -> None:
        """The checked GEMV of this rank's rows; with several ranks, the all-gather of every
        rank's logits and verdicts and their assembly into `logits` (B, V) and `passed`
        (B, checks, V / block). Current stream; no synchronization."""
        self.gemv.launch()
        if self.world > 1:
            self.exchange.gather()
            logits_part, verdict_part = self.exchange.parts
            logits_part.assemble(0, out=self.logits)
            verdict_part.assemble(0, out=self.passed.view(self.batch * self.checks, -1))

    @property
    def gemv_bytes(self) -> int:
        """Algorithmic bytes of this rank's checked GEMV (W, X, logits, bank, verdicts)."""
        return self.gemv.algorithmic_bytes


class TopKTopPSampler:
    """Untrusted top-k / top-p sampler over (B, V) logits with fixed random buffers (graph
    capturable): temperature, the ``k`` largest logits, the shortest prefix of them (in
    descending order) whose probability reaches ``p`` (binary32 softmax, running sum in
    binary32 as a fast sampler computes it), then an inverse-CDF draw. ``fault_rate``
    replaces that share of the tokens (a per-row draw) with the row's lowest logit.

    ``impl``: "kernel" runs `pck_sample_topk_topp` (one launch, one CTA per row; binary32
    logits, k <= 1024), "torch" the same steps as torch operations (topk, softmax, cumsum,
    searchsorted), as the reference's samplers are written."""

    def __init__(self, batch: int, vocab: int, k: int, p: float, temperature: float, device: torch.device,
                 fault_rate: float = 0.0, impl: str = "kernel") -> None:  # fmt: skip
        if not 1 <= k <= vocab or not 0 < p <= 1 or not temperature > 0:
            raise ValueError("need 1 <= k <= V, 0 < p <= 1 and temperature > 0")
        if impl not in ("kernel", "torch") or (impl == "kernel" and k > 1024):
            raise ValueError("impl is 'kernel' (k <= 1024) or 'torch'")
        self.impl, self.vocab = impl, vocab
        self.k, self.p, self.temperature, self.fault_rate = k, p, temperature, fault_rate
        self.draw = torch.empty(batch, dtype=torch.float32, device=device)
        self.fault_draw = torch.empty(batch, dtype=torch.float32, device=device)
        self.tokens = torch.empty(batch, dtype=torch.int64, device=device)
        self.injected = torch.zeros(batch, dtype=torch.bool, device=device)
        self.top_k = torch.full((batch,), k, dtype=torch.int64, device=device)
        self.top_p = torch.full((batch,), p, dtype=torch.float64, device=device)

    def __call__(self, logits: torch.Tensor) -> torch.Tensor:
        self.draw.uniform_()
        if self.impl == "kernel":
            return self._kernel(logits)
        vals, idx = torch.topk(logits / self.temperature, self.k, dim=-1)  # descending
        probs = torch.softmax(vals, dim=-1)
        before = torch.cumsum(probs, dim=-1) - probs
        probs = torch.where(before < self.p, probs, torch.zeros_like(probs))
        cdf = torch.cumsum(probs, dim=-1)
        target = (self.draw * cdf[:, -1]).unsqueeze(-1)
        pick = torch.searchsorted(cdf, target, right=True).clamp(max=self.k - 1)
        # never past the nucleus: the last kept position bounds the pick
        kept = (probs > 0).sum(dim=-1, keepdim=True) - 1
        tokens = idx.gather(-1, torch.minimum(pick, kept)).squeeze(-1)
        if self.fault_rate > 0:
            self.fault_draw.uniform_()
            torch.lt(self.fault_draw, self.fault_rate, out=self.injected)
            tokens = torch.where(self.injected, logits.argmin(dim=-1), tokens)
        self.tokens.copy_(tokens)
        return self.tokens

    def _kernel(self, logits: torch.Tensor) -> torch.Tensor:
        from pck.cuda import _lib
        from pck.cuda._ext import on_device, stream_handle

        if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise RuntimeError("logits must be float32 (B, V) with unit column stride")
        if tuple(logits.shape) != (self.draw.numel(), self.vocab) or logits.device != self.draw.device:
            raise RuntimeError("logits must be (batch, vocab) on the sampler's device")
        faults = None
        if self.fault_rate > 0:
            self.fault_draw.uniform_()
            faults = self.fault_draw.data_ptr()
        else:
            self.injected.zero_()
        with on_device(logits.device):
            rc = _lib.library().pck_sample_topk_topp(
                logits.data_ptr(), logits.size(0), logits.size(1), logits.stride(0), self.k, float(self.p),
                float(self.temperature), self.draw.data_ptr(), faults, float(self.fault_rate),
                self.tokens.data_ptr(), self.injected.data_ptr() if faults else None, stream_handle(logits.device))
        _lib.check(rc, "sampler kernel")
        return self.tokens


def membership(logits: torch.Tensor, sampler: TopKTopPSampler, tol: float = 1e-4) -> dict[str, torch.Tensor]:
    """The fused membership check of the sampler's tokens against the logits it drew from."""
    if sampler.temperature != 1.0:
        logits = logits / sampler.temperature
    return check_members(logits, sampler.tokens, sampler.top_k, sampler.top_p, None, tol)
