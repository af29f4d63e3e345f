"""Kernel-level parity of libmuk against plain PyTorch fp32 restatements.

Each test feeds seeded inputs through one C-ABI entry point and compares
with the same operation computed by torch in fp32 on the same (bf16-rounded)
inputs.  Tolerances are stated per test and sized for bf16 outputs with f32
accumulation.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _kern():
    from mu_b200 import kernels

    return kernels


# ----------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (77, 300, 200), (256, 1024, 4096), (300, 256, 136),
                                   (1024, 8192, 512), (2000, 1152, 256)])
def test_gemm_bf16_and_f32(cuda, M, N, K):
    k = _kern()
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    ref = A.float() @ B.float().t()
    C = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    k.gemm(A, B, C, k.MUK_EPI_BF16)
    # bf16 output: |err| <= 1 bf16 ulp of the value + accumulation noise
    torch.testing.assert_close(C.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())
    Cf = torch.empty(M, N, device=cuda, dtype=torch.float32)
    k.gemm(A, B, Cf, k.MUK_EPI_F32)
    torch.testing.assert_close(Cf, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())


@pytest.mark.parametrize("split", [2, 3, 7])
def test_gemm_split_k(cuda, split):
    k = _kern()
    M, N, K = 200, 384, 1000
    g = torch.Generator(device="cuda").manual_seed(split)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    ref = A.float() @ B.float().t()
    P = torch.full((split, M, N), float("nan"), device=cuda)
    k.gemm(A, B, P, k.MUK_EPI_F32, split_k=split)
    torch.testing.assert_close(P.sum(0), ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())


@pytest.mark.parametrize("I", [256, 192, 1408])
def test_gemm_swiglu_and_bias_silu(cuda, I):
    k = _kern()
    M, K = 130, 320
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    Wg = (torch.randn(I, K, device=cuda, generator=g) * 0.05).bfloat16()
    Wu = (torch.randn(I, K, device=cuda, generator=g) * 0.05).bfloat16()
    # interleave 64-row groups: [g0 u0 g1 u1 ...]
    W = torch.stack([Wg.view(I // 64, 64, K), Wu.view(I // 64, 64, K)], 1).reshape(2 * I, K)
    C = torch.empty(M, I, device=cuda, dtype=torch.bfloat16)
    k.gemm(A, W, C, k.MUK_EPI_SWIGLU)
    gate = A.float() @ Wg.float().t()
    up = A.float() @ Wu.float().t()
    ref = torch.nn.functional.silu(gate) * up
    torch.testing.assert_close(C.float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
    bias = torch.randn(I, device=cuda, generator=g)
    C2 = torch.empty(M, I, device=cuda, dtype=torch.bfloat16)
    k.gemm(A, Wg, C2, k.MUK_EPI_BIAS_SILU, bias=bias)
    ref2 = torch.nn.functional.silu(gate + bias)
    torch.testing.assert_close(C2.float(), ref2, rtol=2e-2, atol=2e-2 * ref2.abs().max().item())


def test_grouped_gemm(cuda):
    k = _kern()
    E, N, K = 4, 256, 192
    counts = [5, 0, 131, 70]
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + c)
    R = offs[-1]
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randn(R, K, device=cuda, generator=g).bfloat16()
    W = (torch.randn(E * N, K, device=cuda, generator=g) * 0.05).bfloat16()
    C = torch.zeros(R, N, device=cuda, dtype=torch.float32)
    off_t = torch.tensor(offs, device=cuda, dtype=torch.int32)
    k.grouped_gemm(A, W, C, off_t, E, N, k.MUK_EPI_F32)
    for e in range(E):
        lo, hi = offs[e], offs[e + 1]
        if hi > lo:
            ref = A[lo:hi].float() @ W[e * N:(e + 1) * N].float().t()
            torch.testing.assert_close(C[lo:hi], ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())


# ----------------------------------------------------------------------------- RoPE + append
def _rope_tables(max_pos, D, theta, device):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2).float() / D))
    t = torch.arange(max_pos).float()
    f = torch.outer(t, inv)
    return f.cos().to(device), f.sin().to(device)


# token-per-CTA layout (D/16 lanes per head, heads of several kinds sharing a
# warp in the small cases) and the warp-per-head fallback (D = 96)
@pytest.mark.parametrize("D,Hq,Hkv,qk_norm", [(128, 32, 8, False), (64, 4, 2, True),
                                              (128, 32, 8, True), (256, 8, 2, True),
                                              (96, 4, 2, True)])
def test_rope_kv_append(cuda, D, Hq, Hkv, qk_norm):
    k = _kern()
    T, NB, bs = 37, 20, 16
    g = torch.Generator(device="cuda").manual_seed(D)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    pos = torch.randint(0, 500, (T,), device=cuda, generator=g, dtype=torch.int32)
    slots = torch.randperm(NB * bs, device=cuda, generator=g)[:T].to(torch.int32)
    slots[3] = -1
    cos, sin = _rope_tables(512, D, 10000.0, cuda)
    kc = torch.zeros(NB, Hkv, bs, D, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    qn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)) if qk_norm else None
    x = qkv.float().clone()
    k.rope_kv_append(qkv, pos, slots, cos, sin, Hq, Hkv, D, kc, vc, qn, kn, 1e-6)

    q = x[:, : Hq * D].view(T, Hq, D)
    kk = x[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = x[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    if qk_norm:
        q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6) * qn
        kk = kk * torch.rsqrt(kk.pow(2).mean(-1, keepdim=True) + 1e-6) * kn
    c = torch.cat([cos, cos], -1)[pos.long()].unsqueeze(1)
    s = torch.cat([sin, sin], -1)[pos.long()].unsqueeze(1)

    def rot(t):
        return torch.cat([-t[..., D // 2:], t[..., : D // 2]], -1)

    q_ref = q * c + rot(q) * s
    k_ref = kk * c + rot(kk) * s
    torch.testing.assert_close(qkv[:, : Hq * D].float().view(T, Hq, D), q_ref, rtol=1e-2, atol=2e-2)
    for t in range(T):
        sl = int(slots[t])
        if sl < 0:
            continue
        blk, off = sl // bs, sl % bs
        torch.testing.assert_close(kc[blk, :, off].float(), k_ref[t], rtol=1e-2, atol=2e-2)
        torch.testing.assert_close(vc[blk, :, off].float(), v[t], rtol=0, atol=0)
    assert k.__name__  # keep the module referenced


# ----------------------------------------------------------------------------- attention
def _build_cache(ctx_lens, Hkv, D, device, seed, extra_blocks=5):
    bs = 16
    nblk = [(c + bs - 1) // bs for c in ctx_lens]
    NB = sum(nblk) + extra_blocks
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(NB, Hkv, bs, D, device=device, generator=g).bfloat16()
    vc = torch.randn(NB, Hkv, bs, D, device=device, generator=g).bfloat16()
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(seed)).tolist()
    maxb = max(nblk)
    bt = torch.zeros(len(ctx_lens), maxb, dtype=torch.int32)
    i = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = torch.tensor(perm[i:i + n], dtype=torch.int32)
        i += n
    return kc, vc, bt.to(device)


def _gather_kv(kc, vc, bt, b, ctx):
    bs = kc.shape[2]
    n = (ctx + bs - 1) // bs
    ids = bt[b, :n].long()
    K = kc[ids].permute(1, 0, 2, 3).reshape(kc.shape[1], n * bs, -1)[:, :ctx]
    V = vc[ids].permute(1, 0, 2, 3).reshape(vc.shape[1], n * bs, -1)[:, :ctx]
    return K.float(), V.float()


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (4, 2, 64), (16, 8, 128)])
def test_paged_decode_attention(cuda, Hq, Hkv, D):
    k = _kern()
    ctx = [1, 15, 16, 17, 33, 300, 2000, 4100, 257, 512]
    kc, vc, bt = _build_cache(ctx, Hkv, D, cuda, seed=Hq + D)
    B = len(ctx)
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn(B, Hq * D, device=cuda, generator=g).bfloat16()
    out = torch.empty_like(q)
    sl = torch.tensor(ctx, dtype=torch.int32, device=cuda)
    max_len = max(ctx)
    ws = torch.empty(k.decode_attn_workspace_size(B, Hq, D, max_len) // 4 + 4, device=cuda)
    k.decode_attn(q, out, kc, vc, bt, sl, Hq, Hkv, D, max_len, workspace=ws)
    G = Hq // Hkv
    for b in range(B):
        K, V = _gather_kv(kc, vc, bt, b, ctx[b])
        qb = q[b].float().view(Hq, D)
        Kr = K.repeat_interleave(G, 0)
        Vr = V.repeat_interleave(G, 0)
        att = torch.softmax((qb.unsqueeze(1) @ Kr.transpose(1, 2)).squeeze(1) / math.sqrt(D), -1)
        ref = (att.unsqueeze(1) @ Vr).squeeze(1)
        torch.testing.assert_close(out[b].float().view(Hq, D), ref, rtol=2e-2, atol=2e-2)


def test_decode_latches_over_long_context(cuda):
    """A context longer than the launch was sized for is skipped with device
    error 5 (bad index) instead of writing past its split slots; the other
    sequences of the batch are unaffected.  Sequence 0 is the long one
    (600 tokens = 38 blocks, 3 splits of 16 against the 2 that max_seq_len 512
    gives), so even its unguarded writes would stay inside this workspace."""
    from mu_b200 import _lib

    k = _kern()
    Hq, Hkv, D = 32, 8, 128
    ctx = [600, 100, 300]
    max_len = 512
    assert _lib.load().muk_decode_attn_splits(len(ctx), max_len, 16) == 2
    kc, vc, bt = _build_cache(ctx, Hkv, D, cuda, seed=17)
    assert bt.shape[1] == 38  # the long row is inside its block-table row
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(len(ctx), Hq * D, device=cuda, generator=g).bfloat16()
    out = torch.zeros_like(q)
    sl = torch.tensor(ctx, dtype=torch.int32, device=cuda)
    ws = torch.empty(k.decode_attn_workspace_size(len(ctx), Hq, D, max_len) // 4 + 4, device=cuda)
    k.decode_attn(q, out, kc, vc, bt, sl, Hq, Hkv, D, max_len, workspace=ws)
    assert _lib.device_error() == 5
    assert bool((out[0] == 0).all())
    G = Hq // Hkv
    for b in (1, 2):
        K, V = _gather_kv(kc, vc, bt, b, ctx[b])
        qb = q[b].float().view(Hq, D)
        att = torch.softmax((qb.unsqueeze(1) @ K.repeat_interleave(G, 0).transpose(1, 2))
                            .squeeze(1) / math.sqrt(D), -1)
        ref = (att.unsqueeze(1) @ V.repeat_interleave(G, 0)).squeeze(1)
        torch.testing.assert_close(out[b].float().view(Hq, D), ref, rtol=2e-2, atol=2e-2)


# one CTA per (query tile, group of G query heads sharing a KV head): G = 4
# (32/8, and 32/4 where two CTAs share a KV head), G = 2 (4/2, 16/8), G = 1
@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (4, 2, 64), (32, 4, 128), (16, 8, 128),
                                      (8, 8, 64)])
def test_paged_prefill_attention(cuda, Hq, Hkv, D):
    k = _kern()
    # (past, q_len): fresh prompts and continuations with a cached prefix
    cases = [(0, 1), (0, 17), (0, 64), (0, 130), (20, 5), (100, 77), (0, 300)]
    ctx = [p + n for p, n in cases]
    kc, vc, bt = _build_cache(ctx, Hkv, D, cuda, seed=3 + D)
    qlens = [n for _, n in cases]
    cu = [0]
    for n in qlens:
        cu.append(cu[-1] + n)
    T = cu[-1]
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(T, Hq * D, device=cuda, generator=g).bfloat16()
    out = torch.empty_like(q)
    k.prefill_attn(q, out, kc, vc, bt, torch.tensor(ctx, dtype=torch.int32, device=cuda),
                   torch.tensor(cu, dtype=torch.int32, device=cuda), max(qlens), Hq, Hkv, D)
    G = Hq // Hkv
    for b, (past, n) in enumerate(cases):
        K, V = _gather_kv(kc, vc, bt, b, ctx[b])
        Kr = K.repeat_interleave(G, 0)
        Vr = V.repeat_interleave(G, 0)
        qb = q[cu[b]:cu[b + 1]].float().view(n, Hq, D).transpose(0, 1)  # [Hq, n, D]
        s = qb @ Kr.transpose(1, 2) / math.sqrt(D)
        qpos = past + torch.arange(n, device=cuda)
        mask = torch.arange(ctx[b], device=cuda)[None, :] <= qpos[:, None]
        s = s.masked_fill(~mask, float("-inf"))
        ref = torch.softmax(s, -1) @ Vr
        got = out[cu[b]:cu[b + 1]].float().view(n, Hq, D).transpose(0, 1)
        torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2)


# ----------------------------------------------------------------------------- norms
def _mu_clamp(x, mu=0.0, lo=-10.0, hi=10.0):
    c, r = (hi + lo) / 2, (hi - lo) / 2
    return mu + torch.tanh((x - mu - c) / r) * r + c


# hidden sizes reach every row-kernel layout: one float4 per thread (512),
# 2 and 4 float4 per thread over 256 threads (2048, 4096), generic loop (320)
@pytest.mark.parametrize("H", [512, 2048, 4096, 320])
def test_residual_rmsnorm_and_embed(cuda, H):
    k = _kern()
    from mu_b200.kernels import Clamp

    T, V, P = 19, 300, 3
    g = torch.Generator(device="cuda").manual_seed(9)
    table = torch.randn(V, H, device=cuda, generator=g).mul(5).bfloat16()
    ids = torch.randint(0, V, (T,), device=cuda, generator=g, dtype=torch.int32)
    resid = torch.empty(T, H, device=cuda)
    cl = Clamp(True, 0.0, -10.0, 10.0)
    k.embed(ids, table, resid, cl)
    ref = _mu_clamp(table.float()[ids.long()])
    torch.testing.assert_close(resid, ref, rtol=1e-5, atol=1e-5)

    parts = torch.randn(P, T, H, device=cuda, generator=g) * 3
    w = 1 + 0.1 * torch.randn(H, device=cuda, generator=g)
    out = torch.empty(T, H, device=cuda, dtype=torch.bfloat16)
    r0 = resid.clone()
    k.residual_rmsnorm(resid, parts, w, 1e-6, out, clamp=cl, clamp_delta=True, clamp_sum=True,
                       clamp_norm=True)
    r_ref = _mu_clamp(r0 + _mu_clamp(parts.sum(0)))
    torch.testing.assert_close(resid, r_ref, rtol=1e-5, atol=1e-4)
    n_ref = _mu_clamp(w * r_ref * torch.rsqrt(r_ref.pow(2).mean(-1, keepdim=True) + 1e-6))
    torch.testing.assert_close(out.float(), n_ref, rtol=1e-2, atol=1e-2)

    rows = torch.tensor([3, 0, 18], device=cuda, dtype=torch.int32)
    out2 = torch.empty(3, H, device=cuda, dtype=torch.bfloat16)
    k.rmsnorm_rows(resid, rows, w, 1e-6, out2, cl)
    torch.testing.assert_close(out2.float(), n_ref[rows.long()], rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("H", [256, 2048, 4096, 320])
def test_inl_dynamics_and_routing(cuda, H):
    k = _kern()
    from mu_b200.kernels import Clamp

    T, E, V = 23, 4, 1000
    g = torch.Generator(device="cuda").manual_seed(4)
    h = torch.randn(T, H, device=cuda, generator=g)
    ctrl = torch.randn(T, 3 * H, device=cuda, generator=g)
    cb = torch.randn(3 * H, device=cuda, generator=g)
    mp = torch.randn(T, H, device=cuda, generator=g) * 0.1
    mu_param = torch.randn(H, device=cuda, generator=g) * 0.1
    v = torch.randn(T, H, device=cuda, generator=g)
    resid = torch.randn(T, H, device=cuda, generator=g)
    router = (torch.randn(E, H, device=cuda, generator=g) * 2).bfloat16()
    ids = torch.randint(0, V, (T,), device=cuda, generator=g, dtype=torch.int32)
    w = torch.ones(H, device=cuda)
    v0, r0 = v.clone(), resid.clone()
    v_bf = torch.empty(T, H, device=cuda, dtype=torch.bfloat16)
    mu_out = torch.empty(T, H, device=cuda, dtype=torch.bfloat16)
    nout = torch.empty(T, H, device=cuda, dtype=torch.bfloat16)
    eids = torch.empty(T, device=cuda, dtype=torch.int32)
    cl = Clamp(True)
    k.inl_dynamics(h, ctrl, cb, mp, mu_param, 0.1, v, v_bf, resid, mu_out, w, 1e-6, nout, ids,
                   router, E, V, eids, cl)
    c = ctrl + cb
    a = torch.sigmoid(c[:, :H])
    b = torch.clamp(torch.nn.functional.softplus(c[:, H:2 * H]), max=2.0)
    gt = torch.sigmoid(c[:, 2 * H:])
    mu_c = mu_param + mp
    vn = torch.clamp(a * v0 - b * (h - mu_c), -10, 10)
    hn = h + 0.1 * gt * vn
    r_ref = r0 + hn
    torch.testing.assert_close(v, vn, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(resid, r_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(mu_out.float(), mu_c, rtol=1e-2, atol=1e-2)
    n_ref = _mu_clamp(r_ref * torch.rsqrt(r_ref.pow(2).mean(-1, keepdim=True) + 1e-6))
    torch.testing.assert_close(nout.float(), n_ref, rtol=1e-2, atol=1e-2)
    logits = torch.nn.functional.one_hot((ids.long() % E), E).float() * 10 + mu_c @ router.float().t()
    # routing is integer output: exact except where two experts tie within f32 noise
    ref_e = logits.argmax(-1).int()
    top2 = logits.topk(2, -1).values
    clear = (top2[:, 0] - top2[:, 1]) > 1e-3
    assert torch.equal(eids[clear], ref_e[clear])
    # the first layer: v_zero reads the incoming velocity as 0 (v's contents ignored)
    vz, rz = torch.full_like(v0, float("nan")), r0.clone()
    vz0, rz0 = torch.zeros_like(v0), r0.clone()
    outs = []
    for vv, rr, flag in ((vz, rz, True), (vz0, rz0, False)):
        nb = torch.empty(T, H, device=cuda, dtype=torch.bfloat16)
        k.inl_dynamics(h, ctrl, cb, mp, mu_param, 0.1, vv, v_bf, rr, mu_out, w, 1e-6, nb, ids,
                       router, E, V, eids, cl, v_zero=flag)
        outs.append((vv.clone(), rr.clone(), nb))
    for x, y in zip(*outs):
        assert torch.equal(x, y)


def test_grouped_gemm_swiglu(cuda):
    k = _kern()
    E, I, K = 4, 192, 256
    counts = [3, 150, 0, 40]
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + c)
    R = offs[-1]
    g = torch.Generator(device="cuda").manual_seed(12)
    A = torch.randn(R, K, device=cuda, generator=g).bfloat16()
    Wg = (torch.randn(E, I, K, device=cuda, generator=g) * 0.05).bfloat16()
    Wu = (torch.randn(E, I, K, device=cuda, generator=g) * 0.05).bfloat16()
    W = torch.cat([torch.stack([Wg[e].view(I // 64, 64, K), Wu[e].view(I // 64, 64, K)], 1)
                   .reshape(2 * I, K) for e in range(E)], 0)
    C = torch.zeros(R, I, device=cuda, dtype=torch.bfloat16)
    k.grouped_gemm(A, W, C, torch.tensor(offs, device=cuda, dtype=torch.int32), E, 2 * I,
                   k.MUK_EPI_SWIGLU)
    for e in range(E):
        lo, hi = offs[e], offs[e + 1]
        if hi > lo:
            ref = (torch.nn.functional.silu(A[lo:hi].float() @ Wg[e].float().t())
                   * (A[lo:hi].float() @ Wu[e].float().t()))
            torch.testing.assert_close(C[lo:hi].float(), ref, rtol=2e-2,
                                       atol=2e-2 * ref.abs().max().item())


def test_route_permute_and_gather(cuda):
    k = _kern()
    T, E = 3000, 8
    g = torch.Generator(device="cuda").manual_seed(8)
    e = torch.randint(0, E, (T,), device=cuda, generator=g, dtype=torch.int32)
    offs = torch.empty(E + 1, device=cuda, dtype=torch.int32)
    perm = torch.empty(T, device=cuda, dtype=torch.int32)
    inv = torch.empty(T, device=cuda, dtype=torch.int32)
    k.route_permute(e, E, offs, perm, inv)
    ref_perm = torch.sort(e.long(), stable=True).indices
    assert torch.equal(perm.long(), ref_perm)
    counts = torch.bincount(e.long(), minlength=E)
    assert torch.equal(offs.long(), torch.cat([torch.zeros(1, device=cuda, dtype=torch.long),
                                               counts.cumsum(0)]))
    assert torch.equal(inv.long()[perm.long()], torch.arange(T, device=cuda))
    src = torch.randn(T, 136, device=cuda, generator=g).bfloat16()
    dst = torch.empty_like(src)
    k.gather_rows(src, perm, dst)
    assert torch.equal(dst, src[perm.long()])


# ----------------------------------------------------------------------------- sampler
def test_sampler_greedy_and_penalty(cuda):
    k = _kern()
    B, V = 6, 5000
    g = torch.Generator(device="cuda").manual_seed(12)
    logits = torch.randn(B, V, device=cuda, generator=g) * 3
    words = (V + 31) // 32
    seen = torch.zeros(B, words, device=cuda, dtype=torch.int32)
    top = logits.argmax(-1)
    # mark each row's argmax as seen so a penalty of 100 dethrones it
    k.mark_seen(seen, torch.arange(B, device=cuda, dtype=torch.int32), top.int(), V)
    zeros = torch.zeros(B, device=cuda)
    out = torch.empty(B, device=cuda, dtype=torch.int32)
    tk = torch.zeros(B, device=cuda, dtype=torch.int32)
    tp = torch.ones(B, device=cuda)
    rp = torch.ones(B, device=cuda)
    seeds = torch.zeros(B, device=cuda, dtype=torch.int64)
    k.sample(logits, zeros, tk, tp, rp, seen, seeds, seeds, out)
    assert torch.equal(out.long(), top)
    rp = torch.full((B,), 100.0, device=cuda)
    k.sample(logits, zeros, tk, tp, rp, seen, seeds, seeds, out)
    pen = logits.clone()
    idx = torch.arange(B, device=cuda)
    v = pen[idx, top]
    pen[idx, top] = torch.where(v > 0, v / 100, v * 100)
    assert torch.equal(out.long(), pen.argmax(-1))


def test_sampler_topk_topp_support_and_distribution(cuda):
    k = _kern()
    V, draws = 1000, 4000
    g = torch.Generator(device="cuda").manual_seed(13)
    base = torch.randn(V, device=cuda, generator=g) * 2
    logits = base.expand(draws, V).contiguous()
    temp, K, P = 0.7, 50, 0.9
    x = base / temp
    kth = x.topk(K).values[-1]
    x = torch.where(x < kth, torch.full_like(x, float("-inf")), x)
    sv, si = torch.sort(x, descending=True)
    cum = torch.softmax(sv, -1).cumsum(-1)
    rm = cum > P
    rm[1:] = rm[:-1].clone()
    rm[0] = False
    allowed = torch.zeros(V, dtype=torch.bool, device=cuda)
    allowed[si[~rm]] = True
    probs = torch.softmax(x.masked_fill(~allowed, float("-inf")), -1)
    out = torch.empty(draws, device=cuda, dtype=torch.int32)
    k.sample(logits, torch.full((draws,), temp, device=cuda),
             torch.full((draws,), K, device=cuda, dtype=torch.int32),
             torch.full((draws,), P, device=cuda), torch.ones(draws, device=cuda), None,
             torch.arange(draws, device=cuda, dtype=torch.int64),
             torch.zeros(draws, device=cuda, dtype=torch.int64), out)
    assert bool(allowed[out.long()].all())
    freq = torch.bincount(out.long(), minlength=V).float() / draws
    # total-variation distance of 4000 draws from the filtered softmax
    assert 0.5 * (freq - probs).abs().sum().item() < 0.08
    # top_k disabled: 1000 survivors, still at most 1024, so this is the exact
    # sorted path again; the radix path runs in test_prepare_logits_large_vocab
    k.sample(logits, torch.full((draws,), temp, device=cuda),
             torch.zeros(draws, device=cuda, dtype=torch.int32),
             torch.full((draws,), P, device=cuda), torch.ones(draws, device=cuda), None,
             torch.arange(draws, device=cuda, dtype=torch.int64),
             torch.zeros(draws, device=cuda, dtype=torch.int64), out)
    x2 = base / temp
    sv, si = torch.sort(x2, descending=True)
    cum = torch.softmax(sv, -1).cumsum(-1)
    rm = cum > P
    rm[1:] = rm[:-1].clone()
    rm[0] = False
    allowed2 = torch.zeros(V, dtype=torch.bool, device=cuda)
    allowed2[si[~rm]] = True
    assert bool(allowed2[out.long()].all())


def _prepare_rows(k, cuda, x, cases, past, V):
    """muk_prepare_logits of one logits row under each (T, top_k, top_p, rp) case."""
    n = len(cases)
    logits = torch.from_numpy(x).to(cuda).expand(n, V).contiguous()
    seen = torch.zeros(n, (V + 31) // 32, device=cuda, dtype=torch.int32)
    if past:
        toks = torch.tensor(past, device=cuda, dtype=torch.int32)
        for r in range(n):
            k.mark_seen(seen, torch.full_like(toks, r), toks, V)
    col = lambda i, dt: torch.tensor([c[i] for c in cases], device=cuda, dtype=dt)  # noqa: E731
    out = torch.empty(n, V, device=cuda)
    k.prepare_logits(logits, col(0, torch.float32), col(1, torch.int32), col(2, torch.float32),
                     col(3, torch.float32), seen, out)
    return out.cpu().numpy(), (logits, seen, col)


def test_prepare_logits_reference_cases(cuda):
    """GPU prepare_logits on the reference-made fixture (V = 1000, exact path):
    same removed set, same kept values."""
    import numpy as np

    import oracle as O  # noqa: F401
    from golden_models import G, top_p_band

    k = _kern()
    d = np.load(G / "sampling.npz")
    cases = [tuple(c) for c in d["cases"]]
    past = d["past"].tolist()
    got, _ = _prepare_rows(k, cuda, d["logits"], cases, past, d["logits"].shape[0])
    for c, (t, kk, p, rp) in enumerate(cases):
        ref = d["out"][c]
        band = top_p_band(d["logits"], t, int(kk), rp, past, p)
        assert np.array_equal(np.isinf(got[c])[~band], np.isinf(ref)[~band]), c
        fin = ~np.isinf(ref) & ~np.isinf(got[c])
        np.testing.assert_allclose(got[c][fin], ref[fin], rtol=1e-6, atol=1e-6)


def test_reference_api_prepare_logits_and_sample_token(cuda):
    """mu_b200.utils.sampling.prepare_logits / sample_token, the reference's
    single-row API (utils/sampling.py:20-120), on a CPU [1, V] tensor: the
    processed logits equal the reference's for every fixture case, and the
    draws of sample_token land in the kept set."""
    import numpy as np

    from golden_models import G, top_p_band
    from mu_b200.utils.sampling import prepare_logits, sample_token

    d = np.load(G / "sampling.npz")
    past = d["past"].tolist()
    x = torch.from_numpy(d["logits"])[None]
    for c, (t, kk, p, rp) in enumerate(d["cases"]):
        got = prepare_logits(x, float(t), int(kk), float(p), float(rp), past)
        assert got.device.type == "cpu" and got.shape == x.shape
        got = got.numpy()[0]
        ref = d["out"][c]
        band = top_p_band(d["logits"], t, int(kk), rp, past, p)
        assert np.array_equal(np.isinf(got)[~band], np.isinf(ref)[~band]), c
        fin = ~np.isinf(ref) & ~np.isinf(got)
        np.testing.assert_allclose(got[fin], ref[fin], rtol=1e-6, atol=1e-6)
        proc = torch.from_numpy(got)[None]
        for s in range(8):
            tok = sample_token(proc, True, seed=s, step=c)
            assert np.isfinite(got[tok]), (c, s, tok)
        assert sample_token(proc, False) == int(np.argmax(got))


def test_prepare_logits_large_vocab(cuda):
    """Radix top-p path (more than 1024 survivors) at V = 32000 and 128256,
    top_k 0 or 2000, top_p 0.5 / 0.9 / 0.99, T 0.7, with and without a
    repetition penalty.  The kept set must equal the reference's outside the
    top-p boundary band (its float32 softmax sum moves the cut; see
    golden_models.TOP_P_BAND) and the oracle's outside a 1e-6 band; kept
    values are bit-identical to the penalised, temperature-scaled logits.
    The draws of muk_sample land in the kept set and repeat exactly."""
    import numpy as np

    import oracle as O
    from golden_models import (G, LARGE_SAMPLING_CASES, LARGE_SAMPLING_VOCABS, large_logits,
                               large_past, top_p_band)

    k = _kern()
    d = np.load(G / "sampling_large.npz")
    cases = list(LARGE_SAMPLING_CASES)
    for V in LARGE_SAMPLING_VOCABS:
        x = large_logits(V)
        past = large_past(V)
        got, (logits, seen, col) = _prepare_rows(k, cuda, x, cases, past, V)
        for c, (t, kk, p, rp) in enumerate(cases):
            ref = np.unpackbits(d[f"masks_{V}"][c])[:V].astype(bool)
            ora = O.prepare_logits(x, t, kk, p, rp, past)
            kept = ~np.isinf(got[c])
            band = top_p_band(x, t, kk, rp, past, p)
            tight = top_p_band(x, t, kk, rp, past, p, 1e-6)
            assert np.array_equal(kept[~band], ref[~band]), (V, c)
            assert np.array_equal(kept[~tight], ~np.isinf(ora)[~tight]), (V, c)
            both = kept & ~np.isinf(ora)
            assert np.array_equal(got[c][both], ora[both]), (V, c)
            # draws: 64 seeds per case, inside the kept set, identical on repeat
            n = 64
            lg = logits[c:c + 1].expand(n, V).contiguous()
            sr = torch.full((n,), c, device=cuda, dtype=torch.int32)
            args = (lg, torch.full((n,), t, device=cuda), torch.full((n,), kk, device=cuda,
                                                                   dtype=torch.int32),
                    torch.full((n,), p, device=cuda), torch.full((n,), rp, device=cuda), seen,
                    torch.arange(n, device=cuda, dtype=torch.int64),
                    torch.full((n,), 5, device=cuda, dtype=torch.int64))
            o1 = torch.empty(n, device=cuda, dtype=torch.int32)
            o2 = torch.empty_like(o1)
            k.sample(*args, o1, seen_rows=sr)
            k.sample(*args, o2, seen_rows=sr)
            assert torch.equal(o1, o2)
            assert kept[o1.cpu().numpy()].all(), (V, c)


def test_no_device_error_left(cuda):
    from mu_b200 import _lib

    assert _lib.device_error() == 0


# Stream-K schedules: shapes whose tile count is not a multiple of the
# workers; the plan is checked so the test cannot pass on a data-parallel
# launch.  (M, N, K, epilogue): tiles < workers with many shares per tile,
# one to two waves, more than two waves (SwiGLU), single-CTA kernel (M <= 128),
# ragged K, bias + SiLU.
SK_CASES = [(256, 4096, 4096, "f32"), (809, 6144, 4096, "bf16"), (809, 28672, 4096, "swiglu"),
            (128, 4096, 4096, "bf16"), (640, 1536, 4000, "f32"), (300, 2816, 2048, "bias_silu")]


@pytest.mark.parametrize("M,N,K,epi", SK_CASES)
def test_gemm_stream_k(cuda, M, N, K, epi):
    k = _kern()
    code = {"f32": k.MUK_EPI_F32, "bf16": k.MUK_EPI_BF16, "swiglu": k.MUK_EPI_SWIGLU,
            "bias_silu": k.MUK_EPI_BIAS_SILU}[epi]
    prev = k.gemm_set_stream_k(1)
    try:
        _check_stream_k(k, cuda, M, N, K, epi, code)
    finally:
        k.gemm_set_stream_k(prev)


def _check_stream_k(k, cuda, M, N, K, epi, code):
    plan = k.gemm_plan_info(M, N, K, code)
    assert plan["stream_k"] == 1 and plan["sk_tiles"] > 0, plan
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    bias = torch.randn(N, device=cuda, generator=g) if epi == "bias_silu" else None
    ref = A.float() @ B.float().t()
    if epi == "swiglu":
        I = N // 2
        gate = ref.view(M, I // 64, 2, 64)[:, :, 0].reshape(M, I)
        up = ref.view(M, I // 64, 2, 64)[:, :, 1].reshape(M, I)
        ref = torch.nn.functional.silu(gate) * up
    elif epi == "bias_silu":
        ref = torch.nn.functional.silu(ref + bias)
    out_dtype = torch.float32 if epi == "f32" else torch.bfloat16
    C = torch.full((M, ref.shape[1]), float("nan"), device=cuda, dtype=out_dtype)
    k.gemm(A, B, C, code, bias=bias)
    tol = 1e-4 if epi == "f32" else 2e-2
    torch.testing.assert_close(C.float(), ref, rtol=tol, atol=tol * ref.abs().max().item())
    # shares are summed in a fixed order: bit-identical on a second launch
    C2 = torch.full_like(C, float("nan"))
    k.gemm(A, B, C2, code, bias=bias)
    assert torch.equal(C, C2)
    from mu_b200 import _lib

    assert _lib.device_error() == 0


def test_decode_workspace_covers_smaller_batches(cuda):
    """A workspace sized for the largest batch must serve every smaller one
    (smaller batches split their contexts more finely)."""
    k = _kern()
    Hq, Hkv, D, bs = 16, 8, 128, 16
    max_len, max_seqs = 672, 64
    ws_bytes = k.decode_attn_workspace_size(max_seqs, Hq, D, max_len)
    ws = torch.empty(max(ws_bytes // 4, 4), device=cuda)
    g = torch.Generator(device="cuda").manual_seed(9)
    for B in (1, 5, 10, 40, 64):
        nb = (max_len + bs - 1) // bs
        kc = torch.randn(B * nb, Hkv, bs, D, device=cuda, generator=g).bfloat16()
        vc = torch.randn(B * nb, Hkv, bs, D, device=cuda, generator=g).bfloat16()
        bt = torch.arange(B * nb, device=cuda, dtype=torch.int32).view(B, nb)
        sl = torch.full((B,), max_len, device=cuda, dtype=torch.int32)
        q = torch.randn(B, Hq * D, device=cuda, generator=g).bfloat16()
        out = torch.empty_like(q)
        k.decode_attn(q, out, kc, vc, bt, sl, Hq, Hkv, D, max_len, workspace=ws)
        Kf = kc.float().permute(0, 2, 1, 3).reshape(B, nb * bs, Hkv, D)[:, :max_len]
        Vf = vc.float().permute(0, 2, 1, 3).reshape(B, nb * bs, Hkv, D)[:, :max_len]
        Kf = Kf.repeat_interleave(Hq // Hkv, 2)
        Vf = Vf.repeat_interleave(Hq // Hkv, 2)
        qf = q.float().view(B, Hq, D)
        att = torch.einsum("bhd,bthd->bht", qf, Kf) / math.sqrt(D)
        ref = torch.einsum("bht,bthd->bhd", att.softmax(-1), Vf).reshape(B, Hq * D)
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


# q|k|v projection with RoPE (+QK-norm) and the KV append in the GEMM epilogue:
# 1-SM and CTA-pair kernels, head_dim 64 and 128, padding slots (-1); the
# last two cases run stream-K schedules (1-SM and pair), whose shares are
# summed into the accumulator before the RoPE epilogue reads it
@pytest.mark.parametrize("M,Hq,Hkv,D,qk_norm,sk", [(37, 4, 2, 64, True, 0),
                                                   (300, 32, 8, 128, False, 0),
                                                   (600, 32, 8, 128, True, 0),
                                                   (130, 16, 8, 128, False, 0),
                                                   (64, 16, 8, 128, True, 1),
                                                   (200, 32, 8, 128, False, 1)])
def test_gemm_qkv_rope(cuda, M, Hq, Hkv, D, qk_norm, sk):
    k = _kern()
    prev = k.gemm_set_stream_k(sk)
    try:
        _check_qkv_rope(k, cuda, M, Hq, Hkv, D, qk_norm, sk)
    finally:
        k.gemm_set_stream_k(prev)


def _check_qkv_rope(k, cuda, M, Hq, Hkv, D, qk_norm, sk):
    K_, NB, bs = (4096 if sk else 512), 64, 16  # stream-K pays over a long K
    N = (Hq + 2 * Hkv) * D
    if sk:
        plan = k.gemm_plan_info(M, N, K_, 4)  # MUK_EPI_ROPE_KV
        assert plan["stream_k"] == 1 and plan["sk_tiles"] > 0, plan
    g = torch.Generator(device="cuda").manual_seed(M + D)
    A = torch.randn(M, K_, device=cuda, generator=g).bfloat16()
    W = (torch.randn(N, K_, device=cuda, generator=g) * 0.05).bfloat16()
    pos = torch.randint(0, 500, (M,), device=cuda, generator=g, dtype=torch.int32)
    slots = torch.randperm(NB * bs, device=cuda, generator=g)[:M].to(torch.int32)
    slots[M // 3] = -1
    cos, sin = _rope_tables(512, D, 10000.0, cuda)
    kc = torch.zeros(NB, Hkv, bs, D, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    qn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)) if qk_norm else None
    q_out = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
    k.gemm_qkv_rope(A, W, q_out, pos, slots, cos, sin, Hq, Hkv, D, kc, vc, qn, kn, 1e-6)
    x = A.float() @ W.float().t()
    q = x[:, : Hq * D].view(M, Hq, D)
    kk = x[:, Hq * D:(Hq + Hkv) * D].view(M, Hkv, D)
    v = x[:, (Hq + Hkv) * D:].view(M, Hkv, D)
    if qk_norm:
        q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6) * qn
        kk = kk * torch.rsqrt(kk.pow(2).mean(-1, keepdim=True) + 1e-6) * kn
    c = torch.cat([cos, cos], -1)[pos.long()].unsqueeze(1)
    s = torch.cat([sin, sin], -1)[pos.long()].unsqueeze(1)

    def rot(t):
        return torch.cat([-t[..., D // 2:], t[..., : D // 2]], -1)

    q_ref = q * c + rot(q) * s
    k_ref = kk * c + rot(kk) * s
    tol = dict(rtol=2e-2, atol=2e-2 * max(1.0, float(q_ref.abs().max())))
    torch.testing.assert_close(q_out[:, : Hq * D].float().view(M, Hq, D), q_ref, **tol)
    for t in range(M):
        sl = int(slots[t])
        if sl < 0:
            continue
        blk, off = sl // bs, sl % bs
        torch.testing.assert_close(kc[blk, :, off].float(), k_ref[t], **tol)
        torch.testing.assert_close(vc[blk, :, off].float(), v[t], **tol)
    # the padding token appended nothing
    from mu_b200 import _lib

    assert _lib.device_error() == 0


# RMSNorm split across two GEMMs: the producer (O / down projection) adds its
# output to the f32 residual and leaves bf16(w * r) plus per-128-column
# partial sums of r^2; the consumer (gate|up or q|k|v) scales each row by
# rsqrt(mean(r^2) + eps).  (M, N, K, stream-K mode): one row, a CTA-pair
# shape, the Llama-3-8B O projection at a mean step, one 128-column part.
@pytest.mark.parametrize("M,N,K,sk", [(1, 512, 384, 0), (130, 1024, 640, 0),
                                      (857, 4096, 4096, 1), (600, 4096, 4096, 0),
                                      (300, 128, 256, 2)])
def test_gemm_residual_norm(cuda, M, N, K, sk):
    k = _kern()
    prev = k.gemm_set_stream_k(sk)
    try:
        g = torch.Generator(device="cuda").manual_seed(M + N)
        A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
        W = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
        r0 = torch.randn(M + 3, N, device=cuda, generator=g) * 2
        w = 1 + 0.1 * torch.randn(N, device=cuda, generator=g)
        resid = r0.clone()
        xbuf = torch.full((M + 3, 2 * N), float("nan"), device=cuda, dtype=torch.bfloat16)
        x = xbuf[:, :N]                                   # row stride 2N, like [x | mu_prev]
        sumsq = torch.full((N // 128, M + 5), float("nan"), device=cuda)
        k.gemm_residual_norm(A, W, resid, w, x, sumsq, M=M)
        ref = r0[:M] + A.float() @ W.float().t()
        torch.testing.assert_close(resid[:M], ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())
        assert torch.equal(resid[M:], r0[M:])            # rows past M untouched
        assert torch.equal(x[:M], (w * resid[:M]).bfloat16())
        assert torch.isnan(xbuf[M:].float()).all() and torch.isnan(xbuf[:, N:].float()).all()
        ss = resid[:M].pow(2).view(M, N // 128, 128).sum(-1).t()
        torch.testing.assert_close(sumsq[:, :M], ss, rtol=1e-5, atol=1e-5 * ss.max().item())
        assert torch.isnan(sumsq[:, M:]).all()
        # without a norm weight: the residual add alone
        resid2 = r0.clone()
        k.gemm_residual_norm(A, W, resid2, None, None, None, M=M)
        assert torch.equal(resid2, resid)
    finally:
        k.gemm_set_stream_k(prev)
    from mu_b200 import _lib

    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,sk", [(1, 0), (300, 0), (809, 1)])
def test_gemm_rownorm_consumers(cuda, M, sk):
    k = _kern()
    H, I, eps = 1024, 1536, 1e-5
    Hq, Hkv, D, NB, bs = 8, 2, 128, 64, 16
    g = torch.Generator(device="cuda").manual_seed(M + 11)
    h = torch.randn(M, H, device=cuda, generator=g) * 3
    w = 1 + 0.1 * torch.randn(H, device=cuda, generator=g)
    xt = (w * h).bfloat16()
    sumsq = torch.zeros(H // 128, M + 7, device=cuda)
    sumsq[:, :M] = h.pow(2).view(M, H // 128, 128).sum(-1).t()
    s = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    a = xt.float() * s                                  # the normed input the consumers see
    rn = k.row_norm(sumsq, H, eps)
    prev = k.gemm_set_stream_k(sk)
    try:
        Wg = (torch.randn(I, H, device=cuda, generator=g) * 0.05).bfloat16()
        Wu = (torch.randn(I, H, device=cuda, generator=g) * 0.05).bfloat16()
        W = torch.stack([Wg.view(I // 64, 64, H), Wu.view(I // 64, 64, H)], 1).reshape(2 * I, H)
        C = torch.empty(M, I, device=cuda, dtype=torch.bfloat16)
        k.gemm_swiglu_rownorm(xt, W, C, rn)
        ref = torch.nn.functional.silu(a @ Wg.float().t()) * (a @ Wu.float().t())
        torch.testing.assert_close(C.float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
        # no row norm: the plain SwiGLU GEMM
        C0 = torch.empty_like(C)
        k.gemm_swiglu_rownorm(xt, W, C0, None)
        C1 = torch.empty_like(C)
        k.gemm(xt, W, C1, k.MUK_EPI_SWIGLU)
        assert torch.equal(C0, C1)

        N = (Hq + 2 * Hkv) * D
        Wq = (torch.randn(N, H, device=cuda, generator=g) * 0.05).bfloat16()
        pos = torch.randint(0, 500, (M,), device=cuda, generator=g, dtype=torch.int32)
        slots = torch.randperm(NB * bs, device=cuda, generator=g)[:M].to(torch.int32)
        cos, sin = _rope_tables(512, D, 10000.0, cuda)
        kc = torch.zeros(NB, Hkv, bs, D, device=cuda, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        q_out = torch.zeros(M, N, device=cuda, dtype=torch.bfloat16)
        k.gemm_qkv_rope(xt, Wq, q_out, pos, slots, cos, sin, Hq, Hkv, D, kc, vc, rownorm=rn)
    finally:
        k.gemm_set_stream_k(prev)
    x = a @ Wq.float().t()
    c = torch.cat([cos, cos], -1)[pos.long()].unsqueeze(1)
    sn = torch.cat([sin, sin], -1)[pos.long()].unsqueeze(1)

    def rope(t):
        return t * c + torch.cat([-t[..., D // 2:], t[..., : D // 2]], -1) * sn

    q_ref = rope(x[:, : Hq * D].view(M, Hq, D))
    k_ref = rope(x[:, Hq * D:(Hq + Hkv) * D].view(M, Hkv, D))
    v_ref = x[:, (Hq + Hkv) * D:].view(M, Hkv, D)
    tol = dict(rtol=2e-2, atol=2e-2 * max(1.0, float(q_ref.abs().max())))
    torch.testing.assert_close(q_out[:, : Hq * D].float().view(M, Hq, D), q_ref, **tol)
    blk, off = (slots // bs).long(), (slots % bs).long()
    torch.testing.assert_close(kc[blk, :, off].float(), k_ref, **tol)
    torch.testing.assert_close(vc[blk, :, off].float(), v_ref, **tol)
    from mu_b200 import _lib

    assert _lib.device_error() == 0


# O projection of the Deep layer with the clamp and both output copies in
# the epilogue: one row, a CTA-pair shape, the C5 step shape.
@pytest.mark.parametrize("M,N,K", [(1, 256, 320), (300, 1024, 640), (2338, 4096, 4096)])
def test_gemm_clamp_dual(cuda, M, N, K):
    k = _kern()
    from mu_b200.kernels import Clamp

    g = torch.Generator(device="cuda").manual_seed(M + N)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    W = (torch.randn(N, K, device=cuda, generator=g) * 0.3).bfloat16()
    for cl in (Clamp(True), Clamp(False)):
        C = torch.full((M + 2, N), float("nan"), device=cuda)
        Cb = torch.full((M + 2, 2 * N), float("nan"), device=cuda, dtype=torch.bfloat16)
        k.gemm_clamp_dual(A, W, C, Cb[:, :N], cl, M=M)
        ref = A.float() @ W.float().t()
        if cl.enabled:
            ref = _mu_clamp(ref)
        torch.testing.assert_close(C[:M], ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())
        assert torch.equal(Cb[:M, :N], C[:M].bfloat16())
        assert torch.isnan(C[M:]).all() and torch.isnan(Cb[M:].float()).all()
        assert torch.isnan(Cb[:, N:].float()).all()
    from mu_b200 import _lib

    assert _lib.device_error() == 0


def test_reduce_bias_silu(cuda):
    """Split-K tail of the INL controller's input layer: the f32 GEMM
    partials summed, bias added, SiLU, bf16."""
    k = _kern()
    T, N, Kd, S = 300, 64, 2048, 6
    g = torch.Generator(device="cuda").manual_seed(21)
    A = torch.randn(T, Kd, device=cuda, generator=g).bfloat16()
    W = (torch.randn(N, Kd, device=cuda, generator=g) * 0.05).bfloat16()
    b = torch.randn(N, device=cuda, generator=g)
    part = torch.empty(S, T, N, device=cuda)
    k.gemm(A, W, part, k.MUK_EPI_F32, split_k=S)
    out = torch.full((T + 1, 2 * N), float("nan"), device=cuda, dtype=torch.bfloat16)
    k.reduce_bias_silu(part, b, out[:, :N], num_rows=T)
    ref = torch.nn.functional.silu(A.float() @ W.float().t() + b)
    torch.testing.assert_close(out[:T, :N].float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
    assert torch.isnan(out[T:].float()).all() and torch.isnan(out[:, N:].float()).all()


def test_tp_greedy_single_rank_slice(cuda):
    """muk_tp_greedy with one rank over a column slice: the argmax of the
    penalised slice (divide positive logits of seen tokens by the penalty,
    multiply the others; lowest index on ties), with global indices."""
    import ctypes

    from mu_b200 import _lib

    B, V, c0, n = 37, 4096, 1024, 2048
    g = torch.Generator(device="cuda").manual_seed(31)
    logits = torch.randn(B, V, device=cuda, generator=g)
    logits[3, c0 + 7] = logits[3, c0 + 900] = 50.0          # tie: lowest index wins
    logits[4, c0:c0 + n] = float("-inf")                      # all -inf: index 0
    words = (V + 31) // 32
    seen = torch.randint(-2**31, 2**31 - 1, (B, words), device=cuda, generator=g, dtype=torch.int32)
    rep = torch.full((B,), 1.3, device=cuda)
    rep[::2] = 1.0
    pairs = torch.zeros(2 * 1 * B * 2, device=cuda, dtype=torch.int32)
    flags = torch.zeros(int(_lib.load().muk_allreduce_flag_bytes()) // 4, device=cuda,
                        dtype=torch.int32)
    out = torch.full((B,), -1, device=cuda, dtype=torch.int32)
    pb = (ctypes.c_void_p * 1)(pairs.data_ptr())
    fb = (ctypes.c_void_p * 1)(flags.data_ptr())
    for _ in range(3):  # the pair buffer alternates by call; the result must not
        out.fill_(-1)
        _lib.call("muk_tp_greedy", logits.data_ptr(), V, B, c0, n, rep.data_ptr(), seen.data_ptr(),
                  words, None, ctypes.addressof(pb), B, ctypes.addressof(fb), 0, 1,
                  out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        idx = torch.arange(V, device=cuda)
        bit = ((seen[:, idx >> 5] >> (idx & 31)) & 1).bool()
        pen = torch.where(bit & (rep[:, None] != 1.0),
                          torch.where(logits > 0, logits / rep[:, None], logits * rep[:, None]),
                          logits)[:, c0:c0 + n]
        ref = pen.argmax(-1) + c0                              # first maximum = lowest index
        ref[4] = 0
        assert torch.equal(out.long(), ref), (out, ref)
    assert _lib.device_error() == 0
