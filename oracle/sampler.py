"""CPU restatement of the reference sampler (test infrastructure only).

`motif/model/sampler.py:151-219` (`Sampler.__call__`): repetition penalty over the tokens
seen in the row (each distinct token once: `torch.unique`), temperature, top-k (keep values
>= the k-th largest), top-p (keep the sorted prefix whose mass before each kept token is
<= p), softmax, multinomial.  Restated in fp32 with the draw made explicit: given a uniform
`u` per row, the token is the first index (in vocabulary order) whose inclusive cumulative
probability exceeds `u`, which is how an inverse-CDF multinomial draw reads a uniform.  Used
only by `tests/` to check the CUDA sampler.

`philox4x32_10` restates the published Philox4x32-10 generator (Salmon, Moraes, Dror and
Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) that the device sampler draws
its uniforms from; it is pinned to the Random123 known-answer vectors in the tests.
"""

from typing import Optional

import torch


_M32 = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    """Ten Philox rounds on a 4-word counter with a 2-word key (pure Python integers)."""
    c = [int(x) & _M32 for x in ctr]
    k = [int(x) & _M32 for x in key]
    for _ in range(10):
        p0 = 0xD2511F53 * c[0]
        p1 = 0xCD9E8D57 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k[0]) & _M32, p1 & _M32, ((p0 >> 32) ^ c[3] ^ k[1]) & _M32, p0 & _M32]
        k = [(k[0] + 0x9E3779B9) & _M32, (k[1] + 0xBB67AE85) & _M32]
    return c


def philox_uniforms(seed: int, offset: int, rows: int) -> torch.Tensor:
    """The device sampler's uniforms: counter (row, 0, offset lo, offset hi), key = seed,
    u = (first word >> 8) / 2^24 (exact in fp32)."""
    out = []
    for r in range(rows):
        w = philox4x32_10([r, 0, offset & _M32, (offset >> 32) & _M32], [seed & _M32, (seed >> 32) & _M32])[0]
        out.append((w >> 8) / 16777216.0)
    return torch.tensor(out, dtype=torch.float32)


def filtered_logits(logits: torch.Tensor, hist: Optional[torch.Tensor], temperature: float,
                    top_k: Optional[int], top_p: Optional[float], repetition_penalty: float) -> torch.Tensor:
    x = logits.float().clone()
    if repetition_penalty != 1.0 and hist is not None:  # sampler.py:168-176
        for i in range(x.shape[0]):
            seen = torch.unique(hist[i])
            vals = x[i, seen]
            x[i, seen] = torch.where(vals > 0, vals / repetition_penalty, vals * repetition_penalty)
    if temperature != 1.0:  # :178-179
        x = x / max(temperature, 1e-5)
    if top_k is not None and top_k > 0:  # :184-187
        k = min(top_k, x.shape[-1])
        kth = torch.topk(x, k)[0][..., -1, None]
        x = x.masked_fill(x < kth, float('-inf'))
    if top_p is not None and 0.0 < top_p < 1.0:  # :189-199; ties at the boundary are all kept here
        p = torch.softmax(x, -1)
        keep = torch.zeros_like(x, dtype=torch.bool)
        for i in range(x.shape[0]):
            # mass of the strictly larger values before each token: the exclusive cumulative
            # mass (float64) at the first sorted position of the token's group of equal values
            xs, order = torch.sort(x[i], descending=True, stable=True)
            ps = p[i][order].double()
            excl = torch.cumsum(ps, 0) - ps
            _, inv, counts = torch.unique_consecutive(xs, return_inverse=True, return_counts=True)
            starts = torch.cumsum(counts, 0) - counts
            before = excl[starts][inv]
            k_sorted = (before <= top_p) & (xs > float('-inf'))
            keep[i, order] = k_sorted
        x = x.masked_fill(~keep, float('-inf'))
    return x


def filtered_probs(logits, hist, temperature, top_k, top_p, repetition_penalty) -> torch.Tensor:
    return torch.softmax(filtered_logits(logits, hist, temperature, top_k, top_p, repetition_penalty), -1)


def sample(logits, hist, temperature, top_k, top_p, repetition_penalty, uniforms: torch.Tensor) -> torch.Tensor:
    """Token per row: first index whose inclusive cumulative probability exceeds u."""
    p = filtered_probs(logits, hist, temperature, top_k, top_p, repetition_penalty)
    c = torch.cumsum(p.double(), -1)
    out = torch.empty(p.shape[0], dtype=torch.int64)
    for i in range(p.shape[0]):
        idx = int(torch.searchsorted(c[i], torch.tensor([float(uniforms[i]) * float(c[i, -1])], dtype=torch.float64),
                                     right=True)[0])
        nz = torch.nonzero(p[i] > 0).flatten()
        out[i] = min(idx, int(nz[-1]))
    return out
