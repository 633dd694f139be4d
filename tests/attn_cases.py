"""Seeded attention workloads shared by the GPU parity tests and the attention benchmark.

`op_level_case` is the op-level tree attention configuration: 32 query / 16 KV heads of 128, a shared prefix of 2048
tokens and 8 branches of 64 tokens, K/V paged in blocks of 64 slots through a shuffled page table, Q/K/V N(0,1) in
BF16, softmax scale 1/sqrt(128), with a global tree mask or a 1024-token sliding window on top of it.
"""
import numpy as np
import torch


def op_level_case(prefix=2048, branches=8, branch=64, hq=32, hk=16, d=128, page=64, seed=0, device='cpu'):
    rng = np.random.default_rng(seed)
    n = prefix + branches * branch
    n_pages_prefix = (prefix + page - 1) // page
    n_pages_branch = (branch + page - 1) // page
    n_pages = n_pages_prefix + branches * n_pages_branch
    perm = rng.permutation(n_pages).astype(np.int32)          # logical page -> physical page
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, hq, d, generator=g).to(torch.bfloat16)
    k_pool = torch.randn(n_pages * page, hk, d, generator=g).to(torch.bfloat16)
    v_pool = torch.randn(n_pages * page, hk, d, generator=g).to(torch.bfloat16)
    # segments: the prefix, then each branch; a branch's key list is the prefix pages plus its own pages
    qo = [0, prefix] + [prefix + (b + 1) * branch for b in range(branches)]
    pages, indptr, last = [], [0], []
    prefix_pages = list(perm[:n_pages_prefix])
    pages += prefix_pages
    indptr.append(len(pages))
    last.append(prefix - (n_pages_prefix - 1) * page)
    for b in range(branches):
        own = list(perm[n_pages_prefix + b * n_pages_branch:n_pages_prefix + (b + 1) * n_pages_branch])
        if prefix % page:
            raise ValueError('the prefix must fill whole pages')
        pages += prefix_pages + own
        indptr.append(len(pages))
        last.append(branch - (n_pages_branch - 1) * page)
    return dict(q=q.to(device), k_pool=k_pool.to(device), v_pool=v_pool.to(device),
                qo_indptr=np.asarray(qo, np.int32), kv_indptr=np.asarray(indptr, np.int32),
                kv_indices=np.asarray(pages, np.int32), last_page_len=np.asarray(last, np.int32),
                page_size=page, hq=hq, hk=hk, d=d, sm_scale=1.0 / np.sqrt(d))


def unmasked_pairs(qo, kv_len, window):
    """Number of visible (query, key) pairs of a causal tree segment list, per query head group: the attention FLOP
    count is 4 * hq * d per pair."""
    total = 0
    for s in range(len(qo) - 1):
        ql = int(qo[s + 1]) - int(qo[s])
        kl = int(kv_len[s])
        for j in range(ql):
            hi = kl - ql + j
            lo = max(0, hi - window + 1) if window > 0 else 0
            total += hi - lo + 1
    return total
