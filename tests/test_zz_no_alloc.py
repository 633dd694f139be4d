"""The entry point that allocates nothing, `morj_gemm_norm_epilogue_noalloc`, against the allocating entry points it
varies (`morj_gemm_bf16_peer` + `morj_peer_reduce` for one rank, scratch allocated by torch).

It exists for callers that may not allocate device memory themselves, such as a process driving this library
through its C-ABI with only the buffers it owns and no right to call cudaMalloc; its scratch is a fixed array
inside the library. Two calls in a row check that the second call is not disturbed by what the first
left in that shared array. Collected last, so a run that stops at its first failure has run every other test."""
import ctypes

import pytest
import torch

from morj_b200 import _native as nat
from morj_b200.tp import exchange_layout, partial_target

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0)


def stream():
    return torch.cuda.current_stream().cuda_stream


def allocating(a, w, mode, x, h, w_a, scalar, w_b, has_next):
    """The same computation through the existing entry points, with torch-allocated exchange buffers."""
    M, K = a.shape
    N = w.shape[0]
    lay = exchange_layout(1, N, M)
    buf = torch.zeros(lay['nbytes'], dtype=torch.uint8, device=DEV)
    d = nat.PeerDesc()
    d.world, d.rank, d.max_blocks, d.hidden = 1, 0, lay['max_blocks'], N
    for name in ('part', 'partials', 'rows'):
        getattr(d, name)[0] = buf.data_ptr() + lay['regions'][name][0]
    d.x[0], d.h[0] = x.data_ptr(), h.data_ptr()
    s = stream()
    nat.call('morj_gemm_bf16_peer', a.data_ptr(), K, w.data_ptr(), K, M, N, K, ctypes.addressof(d), s)
    nat.call('morj_peer_reduce', ctypes.addressof(d), mode, M, w_a.data_ptr(),
             scalar.data_ptr() if scalar is not None else None, w_b.data_ptr(), 1e-6, has_next, 0,
             partial_target(1, 1, N), s)
    torch.cuda.synchronize()
    del buf


def no_alloc(a, w, mode, x, h, w_a, scalar, w_b, has_next):
    M, K = a.shape
    N = w.shape[0]
    nat.call('morj_gemm_norm_epilogue_noalloc', a.data_ptr(), K, w.data_ptr(), K, M, N, K, mode, x.data_ptr(),
             h.data_ptr() if h is not None else None, w_a.data_ptr(),
             scalar.data_ptr() if scalar is not None else None, w_b.data_ptr(), 1e-6, has_next, stream())
    torch.cuda.synchronize()


def test_no_alloc_matches_the_allocating_entry_points_on_two_calls_in_a_row():
    g = torch.Generator(device=DEV).manual_seed(7)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device=DEV, generator=g) * scale).to(torch.bfloat16)
    N = 256
    scalar = torch.tensor([0.75], device=DEV).to(torch.bfloat16)
    # call 1: post-attention epilogue over 300 rows; call 2: post-MLP epilogue over 1000 rows; call 3: fewer rows
    # than the call before it, post-MLP without a next layer (no h: the caller passes NULL)
    for mode, M, K, has_next in ((0, 300, 192, 1), (1, 1000, 320, 1), (1, 200, 320, 0)):
        a, w = rnd(M, K), rnd(N, K, scale=0.1)
        w_a, w_b = (1 + 0.1 * rnd(N)).to(torch.bfloat16), (1 + 0.1 * rnd(N)).to(torch.bfloat16)
        x0 = rnd(M, N)
        x_ref, h_ref = x0.clone(), torch.zeros(M, N, device=DEV, dtype=torch.bfloat16)
        x_new, h_new = x0.clone(), torch.full((M, N), float('nan'), device=DEV, dtype=torch.bfloat16)
        sc = scalar if mode == 1 else None
        allocating(a, w, mode, x_ref, h_ref, w_a, sc, w_b, has_next)
        no_alloc(a, w, mode, x_new, h_new if has_next or mode == 0 else None, w_a, sc, w_b, has_next)
        assert nat.device_error(stream()) == 0
        torch.testing.assert_close(x_new.float(), x_ref.float(), atol=1e-2, rtol=1e-2)
        if has_next or mode == 0:
            torch.testing.assert_close(h_new.float(), h_ref.float(), atol=1e-2, rtol=1e-2)
        else:
            assert torch.isnan(h_new.float()).all()  # nothing wrote h


def test_no_alloc_rejects_more_rows_than_its_fixed_scratch_holds():
    a = torch.zeros(20000, 64, device=DEV, dtype=torch.bfloat16)   # 20000 x 256 x 2 bytes > 8 MiB
    w = torch.zeros(256, 64, device=DEV, dtype=torch.bfloat16)
    x = torch.zeros(20000, 256, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match='projection scratch'):
        no_alloc(a, w, 0, x, x, w[0], None, w[0], 1)
    # few columns, too many row blocks: within the byte limit, beyond the counters
    a = torch.zeros(140000, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(16, 64, device=DEV, dtype=torch.bfloat16)
    x = torch.zeros(140000, 16, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match='row blocks'):
        no_alloc(a, w, 0, x, x, w[0], None, w[0], 1)
