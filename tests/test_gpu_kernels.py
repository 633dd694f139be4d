"""Kernel parity on the GPU, through the C-ABI: each sm_100a kernel against a plain FP32 torch reference of the same
op (GEMMs) or the CPU oracle's restatement of the reference op (`oracle/lean_oracle.py`).

Tolerances: BF16 outputs are compared with `max |got - ref| <= tol * max |ref|` (tol 1e-2 for GEMMs and row ops,
two BF16 ulps of the largest value); attention with the norm-wise relative error `||got - ref|| / ||ref|| <= 2e-2`
(the attention criterion of the tree-prefill parity contract) and 5e-2 elementwise against max |ref|.
"""
import numpy as np
import pytest
import torch

from morj_b200 import _native as nat

pytestmark = pytest.mark.gpu

DEV = 'cuda'


def stream():
    return torch.cuda.current_stream().cuda_stream


def i32(a):
    return torch.as_tensor(np.ascontiguousarray(np.asarray(a, dtype=np.int32)), device=DEV)


def close(got, ref, tol=1e-2):
    got, ref = got.float().cpu(), ref.float().cpu()
    scale = ref.abs().max().item() + 1e-30
    err = (got - ref).abs().max().item()
    assert torch.isfinite(got).all()
    assert err <= tol * scale, f'max err {err:.4g} vs max |ref| {scale:.4g}'


def rel(got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    return ((got - ref).norm() / ref.norm()).item()


@pytest.fixture(autouse=True, scope='module')
def _device():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    nat.lib()
    yield
    assert nat.device_error(stream()) == 0


@pytest.mark.parametrize('M,N,K', [(1, 16, 64), (37, 272, 200), (128, 256, 64), (300, 512, 1024),
                                   (2040, 768, 5376), (517, 5376, 4096), (9, 4096, 5376),
                                   # the 31B shapes: each picks a different tile width (208, 224, 240, 128 / 192)
                                   (2040, 5376, 4096), (2040, 8192, 576), (2040, 6144, 512), (9, 5376, 2048),
                                   (5116, 4096, 256), (8704, 2048, 128)])
def test_gemm_store_matches_fp32_matmul(M, N, K):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    c = torch.full((M, N), float('nan'), device=DEV, dtype=torch.bfloat16)
    nat.call('morj_gemm_bf16', a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), N, M, N, K, nat.EPI_STORE, stream())
    torch.cuda.synchronize()
    close(c, a.float() @ b.float().T)


def test_gemm_strided_operands_and_output():
    M, N, K = 200, 256, 512
    a_full = torch.randn(M, K + 64, device=DEV).to(torch.bfloat16)
    b_full = torch.randn(N + 32, K, device=DEV).to(torch.bfloat16) * 0.05
    c_full = torch.zeros(M, N + 128, device=DEV, dtype=torch.bfloat16)
    a, b = a_full[:, 64:], b_full[32:]
    nat.call('morj_gemm_bf16', a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), c_full.data_ptr(),
             c_full.stride(0), M, N, K, nat.EPI_STORE, stream())
    torch.cuda.synchronize()
    close(c_full[:, :N], a.float() @ b.float().T)
    assert (c_full[:, N:] == 0).all()


@pytest.mark.parametrize('M,F,K', [(5, 128, 256), (300, 1024, 256), (2040, 2048, 1024)])
def test_gemm_geglu_epilogue(M, F, K):
    from morj_b200.lean_core import interleave_glu
    from oracle.lean_oracle import gelu_tanh
    a = torch.randn(M, K, device=DEV).to(torch.bfloat16)
    gate = (torch.randn(F, K, device=DEV) * 0.05).to(torch.bfloat16)
    up = (torch.randn(F, K, device=DEV) * 0.05).to(torch.bfloat16)
    w = interleave_glu(gate, up).contiguous()
    out = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
    nat.call('morj_gemm_bf16', a.data_ptr(), K, w.data_ptr(), K, out.data_ptr(), F, M, 2 * F, K, nat.EPI_GEGLU,
             stream())
    torch.cuda.synchronize()
    g = (a.float() @ gate.float().T).bfloat16().float()
    u = (a.float() @ up.float().T).bfloat16().float()
    close(out, gelu_tanh(g) * u)


@pytest.mark.parametrize('d,hq,hk,has_v', [(64, 4, 2, 1), (64, 4, 2, 0), (128, 32, 16, 1), (128, 32, 16, 0)])
def test_qkv_post_matches_oracle(d, hq, hk, has_v):
    from oracle.lean_oracle import qkv_post, rope_tables
    n = 77
    width = (hq + (2 if has_v else 1) * hk) * d
    qkv = torch.randn(n, width).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d)).to(torch.bfloat16)
    pos = np.random.default_rng(0).integers(0, 9000, n)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
    if not has_v:
        inv[d // 8:] = 0  # proportional partial RoPE: zero frequencies beyond the rotated part
    slots = np.random.default_rng(1).permutation(n + 10)[:n]
    q_out = torch.empty(n, hq, d, device=DEV, dtype=torch.bfloat16)
    kp = torch.zeros(n + 10, hk, d, device=DEV, dtype=torch.bfloat16)
    vp = torch.zeros(n + 10, hk, d, device=DEV, dtype=torch.bfloat16)
    qkv_d, qn_d, kn_d, pos_d, inv_d, sl_d = (qkv.to(DEV), qn.to(DEV), kn.to(DEV), i32(pos), inv.to(DEV),
                                              i32(slots))
    nat.call('morj_qkv_post', qkv_d.data_ptr(), width, n, hq, hk, has_v, d, qn_d.data_ptr(), kn_d.data_ptr(),
             pos_d.data_ptr(), inv_d.data_ptr(), sl_d.data_ptr(), 1e-6, q_out.data_ptr(), kp.data_ptr(), vp.data_ptr(),
             stream())
    torch.cuda.synchronize()
    cos, sin = rope_tables(pos, inv)
    q, k, v = qkv_post(qkv, hq, hk, has_v, d, qn, kn, cos, sin, 1e-6, True)
    close(q_out, q)
    close(kp[torch.as_tensor(slots)], k)
    close(vp[torch.as_tensor(slots)], v)


def _run_attention(case, n_bidir=0, window=0, device_tables=True):
    hq, hk, d = case['hq'], case['hk'], case['d']
    q = case['q'].to(DEV)
    kp, vp = case['k_pool'].to(DEV), case['v_pool'].to(DEV)
    out = torch.full(q.shape, float('nan'), device=DEV, dtype=torch.bfloat16)
    qo = case['qo_indptr']
    work = nat.attention_work(qo, case['kv_indptr'], n_bidir, hq, hk, window, case['page_size'],
                              case.get('last_page_len'))
    nw = len(work) // 2
    assert nw > 0
    last = case.get('last_page_len')
    last_d = i32(last) if last is not None else None
    t = [i32(qo), i32(case['kv_indptr']), i32(case['kv_indices']), i32(work)]
    nat.call('morj_tree_attention', q.data_ptr(), q.shape[0], kp.data_ptr(), vp.data_ptr(), kp.shape[0],
             out.data_ptr(), t[0].data_ptr(),
             t[1].data_ptr(), t[2].data_ptr(), last_d.data_ptr() if last_d is not None else None, len(qo) - 1, n_bidir,
             hq, hk, d, case['page_size'], window, float(case['sm_scale']), t[3].data_ptr(), nw, stream())
    torch.cuda.synchronize()
    return out


def _oracle_attention(case, n_bidir=0, window=0):
    from oracle.lean_oracle import tree_attention
    return tree_attention(case['q'], case['k_pool'], case['v_pool'], case['qo_indptr'], case['kv_indptr'],
                          case['kv_indices'], n_bidir, window, float(case['sm_scale']), case['page_size'],
                          case.get('last_page_len'))


def _tree_case(hq, hk, d, window):
    """A planner-built tree (shared prefix, nested branches) with page size 1 slots, as the engine feeds it."""
    from morj_b200.tree import Tree
    rng = np.random.default_rng(5)
    head = list(rng.integers(0, 50, 150))
    seqs = [head + list(rng.integers(0, 50, n)) for n in (3, 70, 1, 131)]
    seqs.append(seqs[1][:200] + list(rng.integers(0, 50, 9)))
    tree = Tree(seqs)
    need = tree.pass_nodes(range(len(seqs)), set())
    plan = tree.plan_pass(need, list(range(len(seqs))), window if window > 0 else 10**9, 10**9, 10**9, False)
    st = plan['steps'][0]
    kk = 's' if window > 0 else 'g'
    n = len(st['tokens'])
    cap = plan['cap'][kk]
    g = torch.Generator().manual_seed(2)
    q = torch.randn(n, hq, d, generator=g).to(torch.bfloat16)
    kp = torch.randn(cap, hk, d, generator=g).to(torch.bfloat16)
    vp = torch.randn(cap, hk, d, generator=g).to(torch.bfloat16)
    return dict(q=q, k_pool=kp, v_pool=vp, qo_indptr=st['qo_indptr'], kv_indptr=st['kv_indptr_' + kk],
                kv_indices=st['kv_indices_' + kk], page_size=1, hq=hq, hk=hk, d=d, sm_scale=1.0)


@pytest.mark.parametrize('d,hq,hk,window', [(64, 4, 2, 0), (64, 4, 2, 64), (128, 32, 16, 0), (128, 32, 16, 100),
                                            (128, 8, 8, 0), (128, 32, 4, 33)])
def test_tree_attention_on_planner_tables_matches_oracle(d, hq, hk, window):
    case = _tree_case(hq, hk, d, window)
    got = _run_attention(case, window=window)
    ref = _oracle_attention(case, window=window)
    assert rel(got, ref) <= 2e-2
    close(got, ref, 5e-2)


@pytest.mark.parametrize('window', [0, 1024])
def test_op_level_paged_tree_attention(window):
    """The op-level configuration: 2048-token prefix + 8 x 64 branches, pages of 64 through a shuffled page table."""
    from attn_cases import op_level_case
    case = op_level_case()
    got = _run_attention(case, window=window)
    ref = _oracle_attention(case, window=window)
    r = rel(got, ref)
    assert r <= 2e-2, r
    close(got, ref, 5e-2)


def test_bidirectional_image_segments():
    """Leading image-block segments drop the causal bound (block longer and shorter than the window)."""
    from morj_b200.tree import Tree
    rng = np.random.default_rng(9)
    seqs = [list(rng.integers(0, 50, 300)) + list(rng.integers(0, 50, n)) for n in (20, 40)]
    tree = Tree(seqs + [seqs[0][:10], seqs[0][:110], seqs[0][:150], seqs[0][:170]])
    bidir = frozenset(n for n in tree.paths[0] if tree.nodes[n][1] in (10, 150))
    assert len(bidir) == 2
    need = tree.pass_nodes([0, 1], set())
    window = 64
    plan = tree.plan_pass(need, [0, 1], window, 10**9, 10**9, False, bidir=bidir)
    st = plan['steps'][0]
    assert st['n_bidir'] == 2
    g = torch.Generator().manual_seed(4)
    n, cap = len(st['tokens']), plan['cap']['s']
    case = dict(q=torch.randn(n, 4, 64, generator=g).to(torch.bfloat16),
                k_pool=torch.randn(cap, 2, 64, generator=g).to(torch.bfloat16),
                v_pool=torch.randn(cap, 2, 64, generator=g).to(torch.bfloat16), qo_indptr=st['qo_indptr'],
                kv_indptr=st['kv_indptr_s'], kv_indices=st['kv_indices_s'], page_size=1, hq=4, hk=2, d=64,
                sm_scale=0.125)
    got = _run_attention(case, n_bidir=2, window=window)
    ref = _oracle_attention(case, n_bidir=2, window=window)
    assert rel(got, ref) <= 2e-2
    close(got, ref, 5e-2)


@pytest.mark.parametrize('H,n', [(256, 67), (5376, 67), (5376, 2040), (8192, 67)])
def test_row_epilogues_match_oracle(H, n):
    from oracle.lean_oracle import attn_epilogue, mlp_epilogue, rmsnorm
    o = torch.randn(n, H).to(torch.bfloat16)
    x = (torch.randn(n, H) * 3).to(torch.bfloat16)
    wp, wq, wn = [(1 + 0.1 * torch.randn(H)).to(torch.bfloat16) for _ in range(3)]
    sc = torch.tensor([0.75], dtype=torch.bfloat16)
    od, xd, h = o.to(DEV), x.to(DEV).clone(), torch.empty(n, H, device=DEV, dtype=torch.bfloat16)
    wp_d, wq_d = wp.to(DEV), wq.to(DEV)  # kept alive until the kernel has run
    nat.call('morj_attn_epilogue', od.data_ptr(), xd.data_ptr(), h.data_ptr(), wp_d.data_ptr(), wq_d.data_ptr(), n,
             H, 1e-6, stream())
    torch.cuda.synchronize()
    xr, hr = attn_epilogue(o, x, wp, wq, 1e-6)
    close(xd, xr)
    close(h, hr)
    xd2 = x.to(DEV).clone()
    wn_d, sc_d = wn.to(DEV), sc.to(DEV)
    nat.call('morj_mlp_epilogue', od.data_ptr(), xd2.data_ptr(), h.data_ptr(), wp_d.data_ptr(), sc_d.data_ptr(),
             wn_d.data_ptr(), n, H, 1e-6, 1, stream())
    torch.cuda.synchronize()
    xr2, hr2 = mlp_epilogue(o, x, wp, sc, wn, 1e-6)
    close(xd2, xr2)
    close(h, hr2)
    # the last layer's form: no next layer, x written in place, h untouched
    xd3, h_keep = x.to(DEV).clone(), h.clone()
    nat.call('morj_mlp_epilogue', od.data_ptr(), xd3.data_ptr(), h.data_ptr(), wp_d.data_ptr(), sc_d.data_ptr(),
             None, n, H, 1e-6, 0, stream())
    torch.cuda.synchronize()
    assert torch.equal(xd3, xd2) and torch.equal(h, h_keep)
    # embedding + image feature rows + input norm
    V = 1000
    emb = (torch.randn(V, H) * 0.02).to(torch.bfloat16)
    tok = np.random.default_rng(0).integers(0, V, n)
    feats = torch.randn(5, H).to(torch.bfloat16)
    fr = np.full(n, -1)
    fr[[3, 10, 11]] = [0, 4, 2]
    scale = float(torch.tensor(H ** 0.5, dtype=torch.bfloat16))
    xo, ho = torch.empty(n, H, device=DEV, dtype=torch.bfloat16), torch.empty(n, H, device=DEV, dtype=torch.bfloat16)
    emb_d, tok_d, fr_d, f_d = emb.to(DEV), i32(tok), i32(fr), feats.to(DEV)
    nat.call('morj_embed_rmsnorm', tok_d.data_ptr(), fr_d.data_ptr(), f_d.data_ptr(), emb_d.data_ptr(), n, H, scale,
             wn_d.data_ptr(), 1e-6, xo.data_ptr(), ho.data_ptr(), stream())
    torch.cuda.synchronize()
    xe = (emb[torch.as_tensor(tok)].float() * scale).bfloat16().float()
    xe[[3, 10, 11]] = feats[[0, 4, 2]].float()
    close(xo, xe)
    close(ho, rmsnorm(xe, wn, 1e-6))


def test_label_head_matches_oracle():
    from oracle.lean_oracle import label_probs
    H, V = 5376, 3000
    x = torch.randn(6, H).to(torch.bfloat16)
    norm = (1 + 0.1 * torch.randn(H)).to(torch.bfloat16)
    emb = (torch.randn(V, H) * 0.02).to(torch.bfloat16)
    seq_row = [0, 2, 2, 5]
    labels = [[1, 2, 3, 4, 5], [7, 8], list(range(100, 355)), [11, 12, 13]]
    indptr = np.concatenate([[0], np.cumsum([len(l) for l in labels])])
    probs = torch.empty(int(indptr[-1]), device=DEV, dtype=torch.float32)
    xd, nd, ed = x.to(DEV), norm.to(DEV), emb.to(DEV)
    sr, ip, li = i32(seq_row), i32(indptr), i32(np.concatenate(labels))
    nat.call('morj_label_head', xd.data_ptr(), H, sr.data_ptr(), ip.data_ptr(), li.data_ptr(), len(labels),
             nd.data_ptr(), ed.data_ptr(), H, 1e-6, 30.0, probs.data_ptr(), stream())
    torch.cuda.synchronize()
    ref = label_probs([x[r].float() for r in seq_row], norm, emb, labels, 30.0, 1e-6)
    got = probs.cpu().numpy()
    for j, r in enumerate(ref):
        np.testing.assert_allclose(got[indptr[j]:indptr[j + 1]], r, atol=1e-4)
        assert abs(got[indptr[j]:indptr[j + 1]].sum() - 1) < 1e-5


def test_row_gather_scatter_and_reference_geglu():
    from oracle.lean_oracle import geglu
    src = torch.randn(50, 136, device=DEV).to(torch.bfloat16)
    rows = [4, 0, 49, 4]
    dst = torch.empty(4, 136, device=DEV, dtype=torch.bfloat16)
    r = i32(rows)
    nat.call('morj_gather_rows', src.data_ptr(), 136, r.data_ptr(), 4, 136, dst.data_ptr(), 136, stream())
    torch.cuda.synchronize()
    assert torch.equal(dst, src[rows])
    pool = torch.zeros(60, 136, device=DEV, dtype=torch.bfloat16)
    r2 = i32([7, 3, 59])
    nat.call('morj_scatter_rows', src.data_ptr(), 136, r2.data_ptr(), 3, 136, pool.data_ptr(), 136, stream())
    torch.cuda.synchronize()
    assert torch.equal(pool[[7, 3, 59]], src[:3])
    others = [i for i in range(60) if i not in (7, 3, 59)]
    assert (pool[others] == 0).all()
    gu = torch.randn(33, 2 * 200).to(torch.bfloat16)
    out = torch.empty(33, 200, device=DEV, dtype=torch.bfloat16)
    gd = gu.to(DEV)
    nat.call('morj_geglu', gd.data_ptr(), 33, 200, out.data_ptr(), stream())
    torch.cuda.synchronize()
    close(out, geglu(gu))


@pytest.mark.parametrize('force', [0, 0x100, 0x200])
@pytest.mark.parametrize('M,H,d,hq,hk,has_v', [(77, 256, 64, 4, 2, 1), (300, 256, 64, 4, 2, 0),
                                               (2040, 5376, 128, 32, 16, 1), (517, 5376, 128, 32, 16, 0),
                                               (9, 5376, 128, 32, 0, 1), (130, 512, 128, 0, 16, 0)])
def test_fused_qkv_gemm_matches_gemm_then_oracle_head_epilogue(M, H, d, hq, hk, has_v, force):
    """morj_gemm_qkv_rope == BF16 projection followed by the reference head epilogue (`_qkv_post`), with the kernel
    chosen per shape, the SM-pair kernel and the one-CTA kernel."""
    from oracle.lean_oracle import qkv_post, rope_tables
    g = torch.Generator(device=DEV).manual_seed(M + hq)
    rows = (hq + (2 if has_v else 1) * hk) * d
    a = torch.randn(M, H, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(rows, H, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).to(torch.bfloat16)
    pos = np.random.default_rng(M).integers(0, 9000, M)
    inv = (1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))).to(DEV)
    cap = M + 5
    slots = np.random.default_rng(M + 1).permutation(cap)[:M]
    q_out = torch.zeros(M, max(hq, 1), d, device=DEV, dtype=torch.bfloat16)
    kp = torch.zeros(cap, max(hk, 1), d, device=DEV, dtype=torch.bfloat16)
    vp = torch.zeros(cap, max(hk, 1), d, device=DEV, dtype=torch.bfloat16)
    pos_d, sl_d = i32(pos), i32(slots)
    rope = torch.empty(9000, d // 2, 2, device=DEV)
    nat.call('morj_rope_table', inv.data_ptr(), d // 2, 9000, rope.data_ptr(), stream())
    nat.call('morj_gemm_qkv_rope', a.data_ptr(), H, w.data_ptr(), H, M, H, hq, hk, has_v | force, d, qn.data_ptr(),
             kn.data_ptr(), pos_d.data_ptr(), rope.data_ptr(), 9000, sl_d.data_ptr() if hk else None, 1e-6,
             q_out.data_ptr() if hq else None, kp.data_ptr() if hk else None, vp.data_ptr() if hk else None, stream())
    torch.cuda.synchronize()
    proj = (a.float() @ w.float().T).bfloat16().cpu()
    if hq == 0:  # the oracle's column layout always starts with q heads
        proj = torch.cat([torch.zeros(M, 0, dtype=torch.bfloat16), proj], 1)
    cos, sin = rope_tables(pos, inv.cpu())
    q, k, v = qkv_post(proj, hq, hk, has_v, d, qn.cpu(), kn.cpu(), cos, sin, 1e-6, True)
    if hq:
        close(q_out, q)
    if hk:
        close(kp[torch.as_tensor(slots)], k)
        close(vp[torch.as_tensor(slots)], v)


def test_rope_table_matches_torch_cos_sin():
    """morj_rope_table == the reference's FP32 `f.cos()`, `f.sin()` of position x inv_freq (`lean_core.py:636-640`),
    on the device, including the proportional partial table (zero frequencies)."""
    inv = torch.cat([1.0 / (10000 ** (torch.arange(0, 96, 2).float() / 128)), torch.zeros(16)]).to(DEV)
    rows = 70000
    tab = torch.empty(rows, 64, 2, device=DEV)
    nat.call('morj_rope_table', inv.data_ptr(), 64, rows, tab.data_ptr(), stream())
    f = torch.arange(rows, device=DEV, dtype=torch.float32)[:, None] * inv[None]
    torch.testing.assert_close(tab[..., 0], f.cos(), rtol=0, atol=2e-7)
    torch.testing.assert_close(tab[..., 1], f.sin(), rtol=0, atol=2e-7)
    with pytest.raises(ValueError):
        nat.call('morj_rope_table', inv.data_ptr(), 63, 10, tab.data_ptr(), stream())


def test_fused_qkv_position_outside_table_sets_device_error():
    """A position beyond the RoPE table is reported through the device error word and its row is left unwritten."""
    M, H, d, hq, hk = 130, 256, 64, 4, 2
    a = torch.randn(M, H, device=DEV).to(torch.bfloat16)
    w = (torch.randn((hq + 2 * hk) * d, H, device=DEV) * 0.05).to(torch.bfloat16)
    qn = torch.ones(d, device=DEV, dtype=torch.bfloat16)
    inv = (1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))).to(DEV)
    rope = torch.empty(100, d // 2, 2, device=DEV)
    nat.call('morj_rope_table', inv.data_ptr(), d // 2, 100, rope.data_ptr(), stream())
    pos = i32(np.arange(M) % 100)
    pos[77] = 100  # one past the table
    slots = i32(np.arange(M))
    q_out = torch.zeros(M, hq, d, device=DEV, dtype=torch.bfloat16)
    kp = torch.zeros(M, hk, d, device=DEV, dtype=torch.bfloat16)
    vp = torch.zeros(M, hk, d, device=DEV, dtype=torch.bfloat16)
    nat.device_error(stream())
    nat.call('morj_gemm_qkv_rope', a.data_ptr(), H, w.data_ptr(), H, M, H, hq, hk, 1, d, qn.data_ptr(),
             qn.data_ptr(), pos.data_ptr(), rope.data_ptr(), 100, slots.data_ptr(), 1e-6, q_out.data_ptr(),
             kp.data_ptr(), vp.data_ptr(), stream())
    assert nat.device_error(stream()) == 0x301
    assert (q_out[77] == 0).all() and (kp[77] == 0).all() and (vp[77] == 0).all()
    assert (q_out[76] != 0).any()


@pytest.mark.parametrize('force', [0x100, 0x200])
@pytest.mark.parametrize('M,N,K', [(1, 16, 64), (130, 272, 200), (256, 256, 128), (300, 5376, 512),
                                   (2040, 8192, 576), (2040, 5376, 640), (517, 2048, 1024)])
def test_gemm_pair_and_single_kernels(force, M, N, K):
    """The SM-pair kernel (tcgen05.mma.cta_group::2, 2-CTA clusters) and the one-CTA kernel on the same shapes."""
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    c = torch.full((M, N), float('nan'), device=DEV, dtype=torch.bfloat16)
    nat.call('morj_gemm_bf16', a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), N, M, N, K,
             nat.EPI_STORE | force, stream())
    torch.cuda.synchronize()
    close(c, a.float() @ b.float().T)


@pytest.mark.parametrize('force', [0x100, 0x200])
def test_gemm_geglu_pair_and_single(force):
    from morj_b200.lean_core import interleave_glu
    from oracle.lean_oracle import gelu_tanh
    M, F, K = 700, 1024, 512
    a = torch.randn(M, K, device=DEV).to(torch.bfloat16)
    gate = (torch.randn(F, K, device=DEV) * 0.05).to(torch.bfloat16)
    up = (torch.randn(F, K, device=DEV) * 0.05).to(torch.bfloat16)
    w = interleave_glu(gate, up).contiguous()
    out = torch.empty(M, F, device=DEV, dtype=torch.bfloat16)
    nat.call('morj_gemm_bf16', a.data_ptr(), K, w.data_ptr(), K, out.data_ptr(), F, M, 2 * F, K,
             nat.EPI_GEGLU | force, stream())
    torch.cuda.synchronize()
    g = (a.float() @ gate.float().T).bfloat16().float()
    u = (a.float() @ up.float().T).bfloat16().float()
    close(out, gelu_tanh(g) * u)
