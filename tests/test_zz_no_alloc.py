"""The allocation-free decode attention entry point (muk_paged_decode_attn_static).

It serves callers that cannot allocate device memory themselves — a process
whose HBM is already reserved by another allocator, or a serving loop that
must avoid cudaMalloc because it can synchronise the device — by keeping its
split-K scratch in a fixed 16 MiB array inside the library.  This file is
named to be collected last, and it passes both on its own in a fresh process
and after the other tests.

Checks, through the C ABI: two calls in a row (different contexts, so the
second reuses scratch the first left behind) match the workspace-taking
muk_paged_decode_attn within the attention tests' tolerance; both batches
really split (so the static array is written and read); the first call,
which resolves the array's device address, changes neither the caching
allocator's count nor the device's free memory; and a shape needing more
scratch than the array holds is rejected with a clear error.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cache(ctx_lens, Hkv, D, seed):
    bs = 16
    nblk = [(c + bs - 1) // bs for c in ctx_lens]
    NB = sum(nblk) + 3
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(NB, Hkv, bs, D, device="cuda", generator=g).bfloat16()
    vc = torch.randn(NB, Hkv, bs, D, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(seed)).tolist()
    bt = torch.zeros(len(ctx_lens), max(nblk), dtype=torch.int32)
    i = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = torch.tensor(perm[i:i + n], dtype=torch.int32)
        i += n
    return kc, vc, bt.cuda()


def _args(q, out, kc, vc, bt, sl, Hq, Hkv, D, max_len):
    return (q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0), kc.data_ptr(), vc.data_ptr(),
            bt.data_ptr(), bt.stride(0), sl.data_ptr(), sl.numel(), Hq, Hkv, D, 16, kc.shape[0],
            D ** -0.5, max_len)


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (4, 2, 64)])
def test_static_scratch_matches_workspace_entry_point(cuda, Hq, Hkv, D):
    from mu_b200 import _lib

    stream = torch.cuda.current_stream().cuda_stream
    for call, ctx in enumerate(([1, 17, 300, 2100, 4096, 33], [5000, 16, 257, 1])):
        kc, vc, bt = _cache(ctx, Hkv, D, seed=10 * call + D)
        g = torch.Generator(device="cuda").manual_seed(call)
        q = torch.randn(len(ctx), Hq * D, device="cuda", generator=g).bfloat16()
        sl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
        mx = max(ctx)
        need = _lib.load().muk_decode_attn_workspace_size(len(ctx), Hq, D, mx, 16)
        assert 0 < need <= _lib.load().muk_decode_attn_static_scratch_bytes()
        # the launched batch itself splits, so the static array carries partials
        assert _lib.load().muk_decode_attn_splits(len(ctx), mx, 16) > 1
        ws = torch.empty(need // 4 + 4, device="cuda")
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        _lib.call("muk_paged_decode_attn", *_args(q, ref, kc, vc, bt, sl, Hq, Hkv, D, mx),
                  ws.data_ptr(), ws.numel() * 4, stream)
        torch.cuda.synchronize()
        # The workspace call above loaded the library's device code (and with
        # it the static array), so nothing may be allocated from here on.
        alloc0, free0 = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
        _lib.call("muk_paged_decode_attn_static", *_args(q, got, kc, vc, bt, sl, Hq, Hkv, D, mx),
                  stream)
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == alloc0
        assert torch.cuda.mem_get_info()[0] == free0
        torch.testing.assert_close(got.float(), ref.float(), rtol=2e-2, atol=2e-2)
    assert _lib.device_error() == 0


def test_static_scratch_rejects_oversize_shapes(cuda):
    from mu_b200 import _lib

    lib = _lib.load()
    cap = lib.muk_decode_attn_static_scratch_bytes()
    Hq, Hkv, D, B, mx = 32, 8, 128, 1024, 32768
    assert lib.muk_decode_attn_workspace_size(B, Hq, D, mx, 16) > cap
    kc = torch.zeros(4, Hkv, 16, D, device="cuda", dtype=torch.bfloat16)
    q = torch.zeros(B, Hq * D, device="cuda", dtype=torch.bfloat16)
    bt = torch.zeros(B, mx // 16, device="cuda", dtype=torch.int32)
    sl = torch.ones(B, device="cuda", dtype=torch.int32)
    rc = lib.muk_paged_decode_attn_static(*_args(q, q, kc, kc, bt, sl, Hq, Hkv, D, mx),
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MUK_ERR_WORKSPACE
    assert "static" in _lib.last_error()
