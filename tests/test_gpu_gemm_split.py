"""Split tiles of the SM-pair GEMM kernel on the GPU, through the C-ABI: with a workspace registered for the stream
(`morj_gemm_workspace_set`), the tiles of the last waves are cut along K between neighbouring SM pairs. Each
epilogue (store, GeGLU, QKV head epilogue, tensor-parallel partial rows) against the FP32 torch reference (same
tolerance as the other GEMM tests: max |got - ref| <= 1e-2 max |ref|) and against the same call without a
workspace (every tile whole); two launches in a row give identical bits (the flags are back at zero). With at most 16
rows the same workspace serves the weight-streaming kernel (every tile's K range spread over all SMs), checked the
same way against the FP32 reference and the tiled kernels."""
import ctypes

import numpy as np
import pytest
import torch

from morj_b200 import _native as nat

pytestmark = pytest.mark.gpu
DEV = 'cuda'


def stream():
    return torch.cuda.current_stream().cuda_stream


def close(got, ref, tol=1e-2):
    got, ref = got.float().cpu(), ref.float().cpu()
    scale = ref.abs().max().item() + 1e-30
    err = (got - ref).abs().max().item()
    assert torch.isfinite(got).all()
    assert err <= tol * scale, f'max err {err:.4g} vs max |ref| {scale:.4g}'


@pytest.fixture(autouse=True, scope='module')
def _device():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    nat.lib()
    yield
    assert nat.device_error(stream()) == 0


def split_tiles(M, N, bn=256, pairs=74):
    t = -(-M // 256) * -(-N // bn)
    return t > pairs and t % pairs != 0


def run_three(launch):
    """(split, split again, whole): the same launch with the workspace registered twice in a row, then without."""
    ws = nat.GemmWorkspace(DEV)
    ws.register(stream())
    try:
        first = launch()
        second = launch()
    finally:
        ws.close()
    whole = launch()
    assert nat.device_error(stream()) == 0
    return first, second, whole


@pytest.mark.parametrize('M,N,K', [(2040, 5376, 4096), (2040, 5376, 21504), (1000, 5120, 640), (517, 9472, 320),
                                   (2040, 5376, 64), (300, 19200, 192), (2040, 37888, 128)])
def test_split_store(M, N, K):
    assert split_tiles(M, N) or N == 37888  # (37888 = 74 x 2 x 256: whole waves, no cut)
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)

    def launch():
        c = torch.full((M, N), float('nan'), device=DEV, dtype=torch.bfloat16)
        nat.call('morj_gemm_bf16', a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), N, M, N, K, nat.EPI_STORE,
                 stream())
        torch.cuda.synchronize()
        return c
    first, second, whole = run_three(launch)
    assert torch.equal(first, second)
    ref = a.float() @ b.float().T
    close(first, ref)
    close(whole, ref)
    close(first, whole)


def test_split_geglu():
    from morj_b200.lean_core import interleave_glu
    from oracle.lean_oracle import gelu_tanh
    M, F, K = 1000, 3200, 512
    assert split_tiles(M, 2 * F)
    a = torch.randn(M, K, device=DEV).to(torch.bfloat16)
    gate = (torch.randn(F, K, device=DEV) * 0.05).to(torch.bfloat16)
    up = (torch.randn(F, K, device=DEV) * 0.05).to(torch.bfloat16)
    w = interleave_glu(gate, up).contiguous()

    def launch():
        out = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
        nat.call('morj_gemm_bf16', a.data_ptr(), K, w.data_ptr(), K, out.data_ptr(), F, M, 2 * F, K,
                 nat.EPI_GEGLU | 0x100, stream())
        torch.cuda.synchronize()
        return out
    first, second, whole = run_three(launch)
    assert torch.equal(first, second)
    g = (a.float() @ gate.float().T).bfloat16().float()
    u = (a.float() @ up.float().T).bfloat16().float()
    close(first, gelu_tanh(g) * u)
    close(first, whole)


def test_split_qkv_head_epilogue():
    """The fused QKV projection on the pair kernel (256 tiles over 74 pairs): the head epilogue runs once per tile,
    after the tail piece has added the head piece's partial."""
    M, H, d, hq, hk = 2040, 5376, 128, 32, 16
    g = torch.Generator(device=DEV).manual_seed(5)
    rows = (hq + 2 * hk) * d
    assert split_tiles(M, rows)
    a = torch.randn(M, H, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(rows, H, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).to(torch.bfloat16)
    pos = torch.as_tensor(np.random.default_rng(1).integers(0, 4000, M).astype(np.int32), device=DEV)
    slots = torch.as_tensor(np.random.default_rng(2).permutation(M).astype(np.int32), device=DEV)
    inv = (1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))).to(DEV)
    rope = torch.empty(4000, d // 2, 2, device=DEV)
    nat.call('morj_rope_table', inv.data_ptr(), d // 2, 4000, rope.data_ptr(), stream())

    def launch(force=0x100):
        q = torch.zeros(M, hq, d, device=DEV, dtype=torch.bfloat16)
        kp = torch.zeros(M, hk, d, device=DEV, dtype=torch.bfloat16)
        vp = torch.zeros(M, hk, d, device=DEV, dtype=torch.bfloat16)
        nat.call('morj_gemm_qkv_rope', a.data_ptr(), H, w.data_ptr(), H, M, H, hq, hk, 1 | force, d, qn.data_ptr(),
                 qn.data_ptr(), pos.data_ptr(), rope.data_ptr(), 4000, slots.data_ptr(), 1e-6, q.data_ptr(),
                 kp.data_ptr(), vp.data_ptr(), stream())
        torch.cuda.synchronize()
        return torch.cat([q.flatten(), kp.flatten(), vp.flatten()])
    first, second, whole = run_three(launch)
    assert torch.equal(first, second)
    close(first, whole)
    close(first, launch(0x200))  # the one-CTA kernel (never split)


def test_split_peer_partial_rows():
    """The tensor-parallel partial epilogue (one rank): the projection rows reach the part buffer and every row
    block's column count reaches its target once, so the owner's reduce completes with the same rows."""
    from morj_b200.tp import exchange_layout, partial_target
    M, N, K = 2040, 5376, 1024
    assert split_tiles(M, N)
    g = torch.Generator(device=DEV).manual_seed(11)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    w_a = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(torch.bfloat16)
    w_b = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(torch.bfloat16)
    x0 = torch.randn(M, N, device=DEV, generator=g).to(torch.bfloat16)
    lay = exchange_layout(1, N, M)

    def launch():
        buf = torch.zeros(lay['nbytes'], dtype=torch.uint8, device=DEV)
        x, h = x0.clone(), torch.zeros(M, N, device=DEV, dtype=torch.bfloat16)
        d = nat.PeerDesc()
        d.world, d.rank, d.max_blocks, d.hidden = 1, 0, lay['max_blocks'], N
        for name in ('part', 'partials', 'rows'):
            getattr(d, name)[0] = buf.data_ptr() + lay['regions'][name][0]
        d.x[0], d.h[0] = x.data_ptr(), h.data_ptr()
        nat.call('morj_gemm_bf16_peer', a.data_ptr(), K, w.data_ptr(), K, M, N, K, ctypes.addressof(d), stream())
        nat.call('morj_peer_reduce', ctypes.addressof(d), 0, M, w_a.data_ptr(), None, w_b.data_ptr(), 1e-6, 1, 0,
                 partial_target(1, 1, N), stream())
        torch.cuda.synchronize()
        part = buf[lay['regions']['part'][0]:lay['regions']['part'][0] + M * N * 2].view(torch.bfloat16)
        return torch.cat([part.clone(), x.flatten(), h.flatten()])
    first, second, whole = run_three(launch)
    assert torch.equal(first, second)
    close(first[:M * N].view(M, N), a.float() @ w.float().T)
    close(first, whole)


def test_workspace_arguments():
    n = nat.gemm_workspace_bytes()
    buf = torch.empty(n + 512, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        nat.call('morj_gemm_workspace_set', stream(), buf.data_ptr() + 16, n)   # not 256-byte aligned
    with pytest.raises(ValueError):
        nat.call('morj_gemm_workspace_set', stream(), buf.data_ptr(), n - 1)    # too small
    nat.call('morj_gemm_workspace_set', stream(), buf.data_ptr(), n)
    nat.call('morj_gemm_workspace_set', stream(), None, 0)                      # removed again
    nat.call('morj_gemm_workspace_remove', buf.data_ptr())                      # (nothing left to remove)


def skinny_three(launch):
    """(skinny, skinny again, tiled): M <= 16 with the workspace registered, twice, then the one-CTA tiled kernel
    (forced, never the skinny path) on the same stream."""
    ws = nat.GemmWorkspace(DEV)
    ws.register(stream())
    try:
        first = launch(0)
        second = launch(0)
        tiled = launch(0x200)
    finally:
        ws.close()
    assert nat.device_error(stream()) == 0
    return first, second, tiled


# the last layer's O (K 4096) and down (K 21504) shapes at 9 and 1 rows; a partial last tile (N 144) with a ragged
# last k-block (K 4104); one unit on one CTA (128 x 64); 208 tiles of 9 k-blocks (two pieces per tile at most)
@pytest.mark.parametrize('M,N,K', [(9, 5376, 4096), (9, 5376, 21504), (1, 5376, 4096), (16, 4096, 5376),
                                   (9, 144, 4104), (3, 128, 64), (12, 26624, 520)])
def test_skinny_store(M, N, K):
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)

    def launch(force):
        c = torch.full((M, N + 16), float('nan'), device=DEV, dtype=torch.bfloat16)  # ldc > N: the pad stays NaN
        nat.call('morj_gemm_bf16', a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), N + 16, M, N, K,
                 nat.EPI_STORE | force, stream())
        torch.cuda.synchronize()
        return c
    first, second, tiled = skinny_three(launch)
    assert torch.equal(first[:, :N], second[:, :N])
    assert torch.isnan(first[:, N:].float()).all()  # (NaN: compared apart, NaN != NaN)
    ref = a.float() @ b.float().T
    close(first[:, :N], ref)
    close(first[:, :N], tiled[:, :N])


@pytest.mark.parametrize('M,F,K', [(9, 21504, 5376), (5, 384, 200), (16, 1152, 1000)])
def test_skinny_geglu(M, F, K):
    from morj_b200.lean_core import interleave_glu
    from oracle.lean_oracle import gelu_tanh
    g = torch.Generator(device=DEV).manual_seed(M + F + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    gate = (torch.randn(F, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    up = (torch.randn(F, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    w = interleave_glu(gate, up).contiguous()

    def launch(force):
        out = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
        nat.call('morj_gemm_bf16', a.data_ptr(), K, w.data_ptr(), K, out.data_ptr(), F, M, 2 * F, K,
                 nat.EPI_GEGLU | force, stream())
        torch.cuda.synchronize()
        return out
    first, second, tiled = skinny_three(launch)
    assert torch.equal(first, second)
    gv = (a.float() @ gate.float().T).bfloat16().float()
    uv = (a.float() @ up.float().T).bfloat16().float()
    close(first, gelu_tanh(gv) * uv)
    close(first, tiled)
