"""j1_op_attention_noalloc (fixed device scratch, no run-time allocation) against
j1_op_attention through the C ABI: two calls in a row with different batches must
each give the results of the allocating entry point."""
import numpy as np
import pytest

import julia1 as j1

pytestmark = pytest.mark.gpu

H = 768


def _case(torch, lens, seed):
    t = sum(lens)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.uint32)
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = torch.randn((t, 3 * H), generator=g, device="cuda").to(torch.bfloat16)
    return qkv, starts, np.array(lens, np.uint32)


def test_noalloc_matches_attention_twice(torch_cuda):
    torch = torch_cuda
    cases = [(_case(torch, [512, 300, 77, 1], 41), 64), (_case(torch, [1000, 16, 640, 129], 42), -1)]
    refs = []
    for (qkv, starts, lens), window in cases:
        ref = torch.full((qkv.shape[0], H), float("nan"), device="cuda", dtype=torch.bfloat16)
        j1.op_attention(qkv, H, starts, lens, window, ref)
        refs.append(ref)
    torch.cuda.synchronize()
    for rep in range(2):
        for ((qkv, starts, lens), window), ref in zip(cases, refs):
            free0 = torch.cuda.mem_get_info()[0]
            out = torch.full((qkv.shape[0], H), float("nan"), device="cuda", dtype=torch.bfloat16)
            torch.cuda.synchronize()
            free1 = torch.cuda.mem_get_info()[0]
            j1.op_attention_noalloc(qkv, H, starts, lens, window, out)
            free2 = torch.cuda.mem_get_info()[0]
            assert torch.isfinite(out.float()).all()
            # same kernel and tiles: the outputs agree to the last bit (tolerance 0)
            assert (out.float() - ref.float()).abs().max().item() <= 0.0
            if rep == 1:
                assert free2 == free1, (free0, free1, free2)


def test_noalloc_rejects_oversize(torch_cuda):
    torch = torch_cuda
    lens = np.full(8193, 1, np.uint32)  # 8193 one-query tiles > 8192
    starts = np.arange(8193, dtype=np.uint32)
    qkv = torch.zeros((8193, 3 * H), device="cuda", dtype=torch.bfloat16)
    ctx = torch.zeros((8193, H), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(j1.J1Error) as e:
        j1.op_attention_noalloc(qkv, H, starts, lens, -1, ctx)
    assert e.value.status == j1.INVALID_ARG and "8192" in str(e.value)
    assert ctx.abs().max().item() == 0.0
    j1.op_attention_noalloc(qkv[:8192], H, starts[:8192], lens[:8192], -1, ctx)  # exactly at the limit
