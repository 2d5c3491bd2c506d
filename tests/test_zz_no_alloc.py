"""The allocation-free attention entry point (mossgpu_attention_decode_paged_noalloc).

It exists for callers that cannot allocate device memory while they run attention (a
real-time audio callback, or a host whose device memory belongs to another allocator).  Its
scratch is a fixed array inside the library, shared by every call on a device, so this test
calls it twice in a row -- a long multi-chunk batch, then a smaller one that must not see the
first call's leftovers -- and checks each result against the workspace entry point
(mossgpu_attention_decode_paged) on the same inputs, within the attention tests' tolerance.
The file name sorts last so a stop-at-first-failure run has already run everything else.
"""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu
PAGE, HEADS, HD = 16, 12, 64
TOL = 1e-4


def make_case(seed, n_pages, pps, positions):
    import torch
    g = torch.Generator().manual_seed(seed)
    R = len(positions)
    kv = torch.randn(n_pages, 2, HEADS, PAGE, HD, generator=g).half().cuda()
    table = torch.randint(0, n_pages, (R, pps), generator=g, dtype=torch.int32).cuda()
    q = torch.randn(R, HEADS * HD, generator=g).cuda()
    slots = torch.arange(R, dtype=torch.int32).cuda()
    pos = torch.tensor(positions, dtype=torch.int32).cuda()
    return q, kv, table, slots, pos


def with_workspace(L, q, kv, table, slots, pos):
    import torch
    out = torch.full_like(q, float("nan"))
    ws = torch.empty(L.mossgpu_attention_workspace_bytes(q.shape[0]), dtype=torch.uint8, device="cuda")
    rc = L.mossgpu_attention_decode_paged(q.data_ptr(), kv.data_ptr(), table.data_ptr(), table.shape[1],
                                          slots.data_ptr(), pos.data_ptr(), q.shape[0], out.data_ptr(), ws.data_ptr(),
                                          ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.mossgpu_op_last_error()
    return out


def without_alloc(L, q, kv, table, slots, pos):
    import torch
    out = torch.full_like(q, float("nan"))
    rc = L.mossgpu_attention_decode_paged_noalloc(q.data_ptr(), kv.data_ptr(), table.data_ptr(), table.shape[1],
                                                  slots.data_ptr(), pos.data_ptr(), q.shape[0], out.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.mossgpu_op_last_error()
    return out


def test_noalloc_attention_matches_workspace_entry_point_twice():
    import torch
    import moss_b200
    moss_b200.build()
    L = moss_b200.lib()
    first = make_case(11, n_pages=700, pps=300, positions=(4095, 2047, 64, 3000, 17))
    second = make_case(12, n_pages=64, pps=40, positions=(0, 15, 16, 31, 100, 255, 600))
    for case in (first, second):
        got = without_alloc(L, *case)
        want = with_workspace(L, *case)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() <= TOL


def torch_fp32(q, kv, table, slots, pos):
    """The attention of llm.cpp:189-217 (scores q.k / 8, softmax, weighted sum of v) in fp32."""
    import torch
    out = torch.empty_like(q)
    for r in range(q.shape[0]):
        n = int(pos[r]) + 1
        pages = table[int(slots[r]), : (n + PAGE - 1) // PAGE].long()
        k = kv[pages, 0].float().permute(1, 0, 2, 3).reshape(HEADS, -1, HD)[:, :n]
        v = kv[pages, 1].float().permute(1, 0, 2, 3).reshape(HEADS, -1, HD)[:, :n]
        s = (q[r].reshape(HEADS, 1, HD) @ k.transpose(1, 2)) * 0.125
        out[r] = (torch.softmax(s, -1) @ v).reshape(-1)
    return out


def test_noalloc_attention_full_batch_widens_chunks():
    """256 rows (the limit) at up to ~4,000 positions: at the base chunk size the plan would cut
    far more than the array's 341 chunks, so it widens them to fit.  The result must still
    match the workspace entry point and a plain fp32 computation, and no wait may run out."""
    import ctypes
    import numpy as np
    import torch
    import moss_b200
    moss_b200.build()
    L = moss_b200.lib()
    positions = tuple(int(x) for x in np.random.default_rng(21).integers(0, 4000, 256))
    case = make_case(14, n_pages=700, pps=250, positions=positions)
    got = without_alloc(L, *case)
    want = with_workspace(L, *case)
    ref = torch_fp32(*case)
    torch.cuda.synchronize()
    assert torch.isfinite(got).all()
    assert (got - want).abs().max().item() <= TOL
    assert (got - ref).abs().max().item() <= TOL
    code = ctypes.c_int(-1)
    assert L.mossgpu_op_device_status(ctypes.byref(code)) == 0, L.mossgpu_op_last_error()
    assert code.value == 0


def test_noalloc_attention_rejects_batches_over_the_limit():
    import torch
    import moss_b200
    moss_b200.build()
    L = moss_b200.lib()
    q, kv, table, slots, pos = make_case(13, n_pages=8, pps=4, positions=(3,) * 257)
    rc = L.mossgpu_attention_decode_paged_noalloc(q.data_ptr(), kv.data_ptr(), table.data_ptr(), table.shape[1],
                                                  slots.data_ptr(), pos.data_ptr(), 257, q.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and b"exceeds the limit of 256" in L.mossgpu_op_last_error()
