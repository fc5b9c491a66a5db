"""ORACLE — test infrastructure only: seeded synthetic inputs for the parity
tests, the smoke check and the benchmark, with the shapes and distributions of
the workloads the reference is measured on.

Q/K/V/dO are drawn as ``randn`` in the storage shape ``[B, T, H, D]`` and viewed as
BHSD through ``transpose(1, 2)``, as benchmark/precision_check.py:120-130 does;
random masks follow precision_check.py:110-117 (Bernoulli keep with the
``(q, min(q, Tk-1))`` entry forced True).  Generation runs on the CPU with an
explicit ``torch.Generator`` so every machine sees identical bytes.
"""

from __future__ import annotations

import math

import torch


def gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def qkv(B, Tq, Tk, Hq, Hk, D, *, dtype=torch.bfloat16, seed=0, with_dout=True):
    """BHSD views over BTHD storage: (q, k, v, dout or None)."""
    g = gen(seed)
    q = torch.randn((B, Tq, Hq, D), generator=g).to(dtype)
    k = torch.randn((B, Tk, Hk, D), generator=g).to(dtype)
    v = torch.randn((B, Tk, Hk, D), generator=g).to(dtype)
    do = torch.randn((B, Tq, Hq, D), generator=g).to(dtype) if with_dout else None
    t = lambda x: None if x is None else x.transpose(1, 2)
    return t(q), t(k), t(v), t(do)


def random_mask(B, H, Tq, Tk, keep_prob, *, seed=1):
    """Bernoulli(keep_prob) bool mask, diagonal-ish entry forced True
    (benchmark/precision_check.py:110-117)."""
    g = gen(seed)
    m = torch.rand((B, H, Tq, Tk), generator=g) < keep_prob
    qi = torch.arange(Tq)
    m[:, :, qi, torch.clamp(qi, max=Tk - 1)] = True
    return m.contiguous()


def packed_doc_mask(B, T, *, min_len=128, max_len=1024, seed=2):
    """[B, 1, T, T] block-diagonal causal mask over seeded documents whose lengths
    are uniform in [min_len, max_len] (the last one truncated)."""
    g = gen(seed)
    m = torch.zeros((B, 1, T, T), dtype=torch.bool)
    causal = torch.ones((T, T), dtype=torch.bool).tril()
    for b in range(B):
        s = 0
        while s < T:
            n = int(torch.randint(min_len, max_len + 1, (1,), generator=g))
            e = min(T, s + n)
            m[b, 0, s:e, s:e] = causal[: e - s, : e - s]
            s = e
    return m


def alibi_score(B, H, Tq, Tk, *, noise_std=0.5, seed=3):
    """fp32 [B, H, Tq, Tk] = 2^(-8(h+1)/H) * (k - q) + N(0, noise_std^2)."""
    g = gen(seed)
    slopes = torch.tensor([2.0 ** (-8.0 * (h + 1) / H) for h in range(H)]).view(1, H, 1, 1)
    rel = (torch.arange(Tk).view(1, 1, 1, Tk) - torch.arange(Tq).view(1, 1, Tq, 1)).float()
    noise = torch.randn((B, H, Tq, Tk), generator=g) * noise_std
    return (slopes * rel + noise).contiguous()


def fwd_flops(B, Hq, Tq, Tk, D, causal):
    """Reference FLOP convention (benchmark/throughput_check.py:85-92)."""
    return 4.0 * B * Hq * Tq * Tk * D * (0.5 if causal else 1.0)


def fwd_bwd_flops(B, Hq, Tq, Tk, D, causal):
    return 14.0 * B * Hq * Tq * Tk * D * (0.5 if causal else 1.0)


def default_scale(D):
    return 1.0 / math.sqrt(D)


def doc_mask(doc_q, doc_k):
    """Bool mask [B, 1, Tq, Tk] of per-token document ids [B, Tq] / [B, Tk]: keep (q, k)
    iff the ids are equal and not negative (negative = padding)."""
    dq = torch.as_tensor(doc_q)
    dk = torch.as_tensor(doc_k)
    keep = (dq[:, :, None] == dk[:, None, :]) & (dq[:, :, None] >= 0)
    return keep[:, None]


def packed_doc_ids(B, T, *, min_len=128, max_len=1024, pad=0, seed=2):
    """[B, T] int32 document ids of seeded documents with lengths uniform in
    [min_len, max_len] (the last truncated), the final `pad` tokens of every row -1."""
    g = gen(seed)
    ids = torch.full((B, T), -1, dtype=torch.int32)
    for b in range(B):
        s, d = 0, 0
        while s < T - pad:
            n = int(torch.randint(min_len, max_len + 1, (1,), generator=g))
            e = min(T - pad, s + n)
            ids[b, s:e] = d
            s, d = e, d + 1
    return ids
