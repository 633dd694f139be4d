"""The peer-memory exchange kernels of tensor parallelism on one GPU (`morj_gemm_bf16_peer`, `morj_peer_reduce`,
`morj_peer_wait`), with the ranks of a group emulated in one process: every rank's buffers are plain allocations
on this GPU, and each site launches all ranks' GEMMs, then all reduces, then all waits, on one stream, so every
wait is already satisfied when it starts (no kernel waits on a kernel running beside it). Checked against the
replicated path: the sum of the delivered partials through `morj_attn_epilogue` / `morj_mlp_epilogue`."""
import ctypes

import numpy as np
import pytest
import torch

from morj_b200 import _native as nat
from morj_b200.tp import BLOCK, exchange_layout, owner, partial_target, row_target

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def stream():
    return torch.cuda.current_stream().cuda_stream


class Group:
    """`world` emulated ranks' exchange buffers on this GPU and their descriptors."""

    def __init__(self, world, hidden, max_rows):
        self.world, self.hidden = world, hidden
        self.lay = exchange_layout(world, hidden, max_rows)
        self.bufs = [torch.zeros(self.lay['nbytes'], dtype=torch.uint8, device=DEV) for _ in range(world)]
        self.descs = []
        for r in range(world):
            d = nat.PeerDesc()
            d.world, d.rank, d.max_blocks, d.hidden = world, r, self.lay['max_blocks'], hidden
            for q in range(world):
                for name, (off, _) in self.lay['regions'].items():
                    getattr(d, name)[q] = self.bufs[q].data_ptr() + off
            self.descs.append(d)
        self.sites = 0

    def region(self, r, name, rows):
        off, _ = self.lay['regions'][name]
        return self.bufs[r][off:off + rows * self.hidden * 2].view(torch.bfloat16).view(rows, self.hidden)

    def delivered(self, n):
        """Every rank's partial rows [0, n): [world, n, hidden], read from their part buffers."""
        return torch.stack([self.region(r, 'part', n) for r in range(self.world)])

    def site(self, a, w, mode, n, w_a, scalar, w_b, has_next, push_x):
        s = stream()
        for r in range(self.world):
            nat.call('morj_gemm_bf16_peer', a[r].data_ptr(), a[r].stride(0), w[r].data_ptr(), w[r].stride(0), n,
                     self.hidden, a[r].shape[1], ctypes.addressof(self.descs[r]), s)
        self.sites += 1
        for r in range(self.world):
            nat.call('morj_peer_reduce', ctypes.addressof(self.descs[r]), mode, n, w_a.data_ptr(),
                     scalar.data_ptr() if scalar is not None else None, w_b.data_ptr(), 1e-6, has_next, push_x,
                     partial_target(self.sites, self.world, self.hidden), s)
        for r in range(self.world):
            nat.call('morj_peer_wait', ctypes.addressof(self.descs[r]), n, row_target(self.sites), s)


def norm_weight(g, hidden):
    return (1 + 0.1 * torch.randn(hidden, device=DEV, generator=g)).to(torch.bfloat16)


@pytest.mark.parametrize('world', [1, 2, 3, 4, 6, 8])  # the reduce kernel's rank bound W = 2, 4, 8
def test_peer_sites_match_the_replicated_epilogues(world):
    hidden, max_rows, k = 256, 1100, 96
    g = torch.Generator(device=DEV).manual_seed(world)
    grp = Group(world, hidden, max_rows)
    x0 = torch.randn(max_rows, hidden, device=DEV, generator=g).to(torch.bfloat16)
    for r in range(world):
        grp.region(r, 'x', max_rows).copy_(x0)
    x_ref = x0.clone()
    h_ref = torch.zeros(max_rows, hidden, device=DEV, dtype=torch.bfloat16)
    w_post, w_pre, w_next = norm_weight(g, hidden), norm_weight(g, hidden), norm_weight(g, hidden)
    scalar = torch.tensor([0.75], device=DEV).to(torch.bfloat16)
    # (mode, rows, has_next, push_x): row counts change between sites, so blocks are padded and then used
    sites = [(0, 300, 1, 0), (1, 300, 1, 0), (0, 1100, 1, 0), (1, 1100, 1, 1), (0, 129, 1, 0), (1, 129, 0, 1),
             (0, 1, 1, 0), (1, 1000, 1, 0)]
    for mode, n, has_next, push_x in sites:
        a = [torch.randn(n, k, device=DEV, generator=g).to(torch.bfloat16) for _ in range(world)]
        w = [(torch.randn(hidden, k, device=DEV, generator=g) * 0.1).to(torch.bfloat16) for _ in range(world)]
        grp.site(a, w, mode, n, w_post, scalar if mode == 1 else None, w_pre if mode == 0 else w_next, has_next,
                 push_x)
        torch.cuda.synchronize()
        assert nat.device_error(stream()) == 0
        parts = grp.delivered(n)
        for r in range(world):  # each delivered partial is that rank's BF16 projection
            torch.testing.assert_close(parts[r].float(), a[r].float() @ w[r].float().T, atol=2e-2, rtol=2e-2)
        acc = parts[0].float()
        for r in range(1, world):
            acc = acc + parts[r].float()
        o = acc.to(torch.bfloat16).contiguous()
        s = stream()
        if mode == 0:
            nat.call('morj_attn_epilogue', o.data_ptr(), x_ref.data_ptr(), h_ref.data_ptr(), w_post.data_ptr(),
                     w_pre.data_ptr(), n, hidden, 1e-6, s)
        else:
            nat.call('morj_mlp_epilogue', o.data_ptr(), x_ref.data_ptr(), h_ref.data_ptr(), w_post.data_ptr(),
                     scalar.data_ptr(), w_next.data_ptr(), n, hidden, 1e-6, has_next, s)
        torch.cuda.synchronize()
        for r in range(world):
            xr = grp.region(r, 'x', max_rows)
            own = np.array([owner(i // BLOCK, world) == r for i in range(n)])
            rows = np.arange(n) if push_x else np.flatnonzero(own)
            assert torch.equal(xr[rows], x_ref[rows]), (mode, n, r)
            if mode == 0 or has_next:
                assert torch.equal(grp.region(r, 'h', max_rows)[:n], h_ref[:n]), (mode, n, r)


def test_peer_waits_run_out_and_report():
    """A partial or row target that no rank will reach: the kernels give up after their bounded wait (2 s), report
    through the device error word (0x104 partials, 0x105 rows) and leave the context usable."""
    hidden = 256
    grp = Group(1, hidden, 256)
    w = norm_weight(torch.Generator(device=DEV).manual_seed(0), hidden)
    s = stream()
    nat.device_error(s)
    d = ctypes.addressof(grp.descs[0])
    nat.call('morj_peer_reduce', d, 0, 200, w.data_ptr(), None, w.data_ptr(), 1e-6, 1, 0,
             partial_target(1, 1, hidden), s)
    assert nat.device_error(s) == 0x104
    nat.call('morj_peer_wait', d, 200, row_target(1), s)
    assert nat.device_error(s) == 0x105
    a = torch.randn(64, 64, device=DEV).to(torch.bfloat16)
    c = torch.empty(64, 64, device=DEV, dtype=torch.bfloat16)
    nat.call('morj_gemm_bf16', a.data_ptr(), 64, a.data_ptr(), 64, c.data_ptr(), 64, 64, 64, 64, 0, s)
    torch.cuda.synchronize()
    torch.testing.assert_close(c.float(), a.float() @ a.float().T, atol=5e-2, rtol=2e-2)
    assert nat.device_error(s) == 0


def test_peer_arguments_are_checked():
    grp = Group(2, 256, 256)
    d = ctypes.addressof(grp.descs[0])
    a = torch.zeros(300, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # more rows than the buffers hold
        nat.call('morj_gemm_bf16_peer', a.data_ptr(), 64, a.data_ptr(), 64, 300, 256, 64, d, stream())
    with pytest.raises(ValueError):  # N must be the exchange's hidden size
        nat.call('morj_gemm_bf16_peer', a.data_ptr(), 64, a.data_ptr(), 64, 200, 128, 64, d, stream())
    grp.descs[0].part[1] = None
    with pytest.raises(ValueError):
        nat.call('morj_peer_wait', d, 10, 0, stream())
