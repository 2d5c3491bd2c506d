"""The standalone paged flash-decode op (mossgpu_attention_decode_paged) against a plain
PyTorch fp32 reference of the same attention (llm.cpp:189-217 semantics) on device buffers."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
PAGE, HEADS, HD = 16, 12, 64


def paged_case(seed=0, n_pages=96, pps=48, positions=(0, 15, 16, 31, 100, 700)):
    import torch
    g = torch.Generator().manual_seed(seed)
    R = len(positions)
    kv = torch.randn(n_pages, 2, HEADS, PAGE, HD, generator=g).half()
    perm = torch.randint(0, n_pages, (R, pps), generator=g, dtype=torch.int32)  # rows may share pages
    q = torch.randn(R, HEADS * HD, generator=g)
    slots = torch.arange(R, dtype=torch.int32)
    pos = torch.tensor(positions, dtype=torch.int32)
    return q, kv, perm, slots, pos


def torch_reference(q, kv, table, slots, pos):
    import torch
    out = torch.empty_like(q)
    for r in range(q.shape[0]):
        n = int(pos[r]) + 1
        pages = table[int(slots[r]), : (n + PAGE - 1) // PAGE].long()
        k = kv[pages, 0].float().permute(1, 0, 2, 3).reshape(HEADS, -1, HD)[:, :n]  # [H][n][64]
        v = kv[pages, 1].float().permute(1, 0, 2, 3).reshape(HEADS, -1, HD)[:, :n]
        qh = q[r].reshape(HEADS, 1, HD)
        s = (qh @ k.transpose(1, 2)) * 0.125
        out[r] = (torch.softmax(s, -1) @ v).reshape(-1)
    return out


@pytest.fixture(scope="module")
def lib():
    import moss_b200
    moss_b200.build()
    return moss_b200.lib()


def call(lib, q, kv, table, slots, pos, ws_bytes=None, stream=None):
    import torch
    R = q.shape[0]
    out = torch.full_like(q, float("nan"))
    need = lib.mossgpu_attention_workspace_bytes(R)
    ws = torch.empty(ws_bytes if ws_bytes is not None else need, dtype=torch.uint8, device="cuda")
    rc = lib.mossgpu_attention_decode_paged(q.data_ptr(), kv.data_ptr(), table.data_ptr(), table.shape[1],
                                            slots.data_ptr(), pos.data_ptr(), R, out.data_ptr(), ws.data_ptr(),
                                            ws.numel(), stream)
    torch.cuda.synchronize()
    return rc, out


def test_attention_op_matches_torch_fp32(lib):
    import torch
    q, kv, table, slots, pos = paged_case()
    ref = torch_reference(q, kv, table, slots, pos)
    dev = [t.cuda() for t in (q, kv, table, slots, pos)]
    s = torch.cuda.current_stream().cuda_stream
    rc, out = call(lib, *dev, stream=s)
    assert rc == 0, lib.mossgpu_op_last_error()
    assert torch.isfinite(out).all()
    assert (out.cpu() - ref).abs().max().item() < 1e-4


def test_attention_op_long_rows_use_many_chunks(lib):
    import torch
    q, kv, table, slots, pos = paged_case(seed=3, n_pages=700, pps=300, positions=(4095, 2047, 64, 3000))
    ref = torch_reference(q, kv, table, slots, pos)
    rc, out = call(lib, *[t.cuda() for t in (q, kv, table, slots, pos)])
    assert rc == 0, lib.mossgpu_op_last_error()
    assert (out.cpu() - ref).abs().max().item() < 1e-4


def test_attention_op_many_ragged_rows(lib):
    # more rows than one 32-row search step, rows of one position next to rows of many
    # chunks, and several chunks handed to every CTA
    import torch
    rng = np.random.default_rng(11)
    positions = tuple(int(x) for x in rng.integers(0, 2000, 150)) + (0, 1, 15, 16, 17)
    q, kv, table, slots, pos = paged_case(seed=5, n_pages=400, pps=128, positions=positions)
    ref = torch_reference(q, kv, table, slots, pos)
    rc, out = call(lib, *[t.cuda() for t in (q, kv, table, slots, pos)])
    assert rc == 0, lib.mossgpu_op_last_error()
    assert torch.isfinite(out).all()
    assert (out.cpu() - ref).abs().max().item() < 1e-4


def test_attention_op_rejects_small_workspace(lib):
    q, kv, table, slots, pos = [t.cuda() for t in paged_case()]
    rc, _ = call(lib, q, kv, table, slots, pos, ws_bytes=64)
    assert rc != 0 and b"workspace" in lib.mossgpu_op_last_error()
