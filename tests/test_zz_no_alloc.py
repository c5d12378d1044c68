"""j1_op_attention_noalloc (fixed device scratch, no run-time allocation) against
j1_op_attention through the C ABI. The entry point is for callers that cannot allocate
device memory (a serving process whose pool already owns the free HBM, or a loop that
must not pay cudaMalloc's device-wide synchronisation): two calls in a row with
different batches must each give the results of the allocating entry point, also when
both are issued asynchronously on one stream, and a device-side timeout of an
asynchronous call must reach the caller through the next synchronous one."""
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


def _cases_and_refs(torch):
    cases = [(_case(torch, [512, 300, 77, 1], 41), 64), (_case(torch, [1000, 16, 640, 129], 42), -1)]
    refs = []
    for (qkv, starts, lens), window in cases:
        ref = torch.full((qkv.shape[0], H), float("nan"), device="cuda", dtype=torch.bfloat16)
        j1.op_attention(qkv, H, starts, lens, window, ref)
        refs.append(ref)
    torch.cuda.synchronize()
    return cases, refs


def test_noalloc_matches_attention_twice(torch_cuda):
    torch = torch_cuda
    cases, refs = _cases_and_refs(torch)
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


def test_noalloc_async_calls_on_one_stream(torch_cuda):
    """Both batches issued with sync=0 on one user stream, one synchronisation at the end:
    the second call's tile upload is ordered after the first call's kernel."""
    torch = torch_cuda
    cases, refs = _cases_and_refs(torch)
    s = torch.cuda.Stream()
    outs = [torch.full((c[0][0].shape[0], H), float("nan"), device="cuda", dtype=torch.bfloat16) for c in cases]
    torch.cuda.synchronize()
    for rep in range(2):
        for ((qkv, starts, lens), window), out in zip(cases, outs):
            j1.op_attention_noalloc(qkv, H, starts, lens, window, out, stream=s.cuda_stream, sync=False)
        s.synchronize()
        for out, ref in zip(outs, refs):
            assert (out.float() - ref.float()).abs().max().item() <= 0.0
        for out in outs:
            out.fill_(float("nan"))
        torch.cuda.synchronize()
    j1.op_attention_noalloc(cases[0][0][0], H, [], [], -1, outs[0], stream=s.cuda_stream, sync=True)  # collects: clean


def test_noalloc_async_timeout_reported_by_next_sync_call(torch_cuda):
    """A device-side timeout in a sync=0 call (a bounded wait that is made to run out, no
    fault) is reported by the next sync=1 call on the device and then cleared."""
    torch = torch_cuda
    cases, refs = _cases_and_refs(torch)
    (qkv, starts, lens), window = cases[0]
    out = torch.zeros((qkv.shape[0], H), device="cuda", dtype=torch.bfloat16)
    j1.inject_fault(j1.FAULT_DEVICE_WAIT, 1)
    try:
        j1.op_attention_noalloc(qkv, H, starts, lens, window, out, sync=False)  # returns before its kernel runs
    finally:
        j1.inject_fault(j1.FAULT_DEVICE_WAIT, 0)
    with pytest.raises(j1.J1Error) as e:
        j1.op_attention_noalloc(qkv, H, [], [], -1, out, sync=True)  # nseq = 0: only collects
    assert e.value.status == j1.DEVICE_TIMEOUT
    assert "earlier call made with sync = 0" in str(e.value) and "site 99" in str(e.value)
    # reported once: the words are clear again and the next calls compute as before
    out.fill_(float("nan"))
    j1.op_attention_noalloc(qkv, H, starts, lens, window, out, sync=True)
    assert (out.float() - refs[0].float()).abs().max().item() <= 0.0
    # the same fault in a sync=1 call is that call's own timeout
    j1.inject_fault(j1.FAULT_DEVICE_WAIT, 1)
    try:
        with pytest.raises(j1.J1Error) as e:
            j1.op_attention_noalloc(qkv, H, starts, lens, window, out, sync=True)
    finally:
        j1.inject_fault(j1.FAULT_DEVICE_WAIT, 0)
    assert e.value.status == j1.DEVICE_TIMEOUT and "earlier" not in str(e.value)
    j1.op_attention_noalloc(qkv, H, starts, lens, window, out, sync=True)


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
