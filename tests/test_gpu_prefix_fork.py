"""Device-side prefix sharing (mossgpu_stream_fork; snapshot_prefix / restore_prefix,
llm.cpp:455-483): a fork shares the source's full KV pages and copies the partial one, steps
exactly like a stream prefilled from scratch, never writes into the source (copy on write),
and its pages go back to the pool once the last stream using them closes."""
from __future__ import annotations

import numpy as np
import pytest

from golden_inputs import forced_codes, prompt_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pkg():
    import moss_b200
    moss_b200.build()
    return moss_b200


@pytest.fixture(scope="module")
def eng(pkg, weights_path):
    e = pkg.Engine(weights_path, device=0, max_streams=8, max_ctx=256)
    yield e
    e.close()


def kv_all(e, s, n):
    return [e.kv(s, layer, 0, n) for layer in range(12)]


def test_fork_shares_the_prefix_and_steps_like_a_fresh_prefill(pkg, eng):
    e = eng
    rows = prompt_rows(40, seed=3)
    a, d = e.open(), e.open()
    e.prefill(a, rows)
    e.prefill(d, rows)
    before = kv_all(e, a, 40)
    b, c = e.fork(a, 40), e.fork(a, 37)  # at a page boundary and inside a page
    try:
        assert e.position(b) == 40 and e.position(c) == 37
        for layer in range(12):
            kb, vb = e.kv(b, layer, 0, 40)
            kc, vc = e.kv(c, layer, 0, 37)
            assert np.array_equal(kb, before[layer][0]) and np.array_equal(vb, before[layer][1])
            assert np.array_equal(kc, before[layer][0][:37]) and np.array_equal(vc, before[layer][1][:37])
        assert np.array_equal(e.hidden(b), e.hidden(a))
        p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=99)
        forced = forced_codes(4, seed=5)
        e.generate_begin(b, 0)
        e.generate_begin(d, 0)
        for f in range(4):
            cb, _, gb, lb = e.step([b], p, forced=forced[f], want_logits=True)
            cd, _, gd, ld = e.step([d], p, forced=forced[f], want_logits=True)
            assert np.array_equal(lb, ld) and np.array_equal(cb, cd) and np.array_equal(gb, gd)
        assert e.position(b) == 44 and e.position(a) == 40
        after = kv_all(e, a, 40)
        for layer in range(12):  # the source's positions are untouched by b's frames
            assert np.array_equal(after[layer][0], before[layer][0])
            assert np.array_equal(after[layer][1], before[layer][1])
    finally:
        for s in (a, b, c, d):
            e.close_stream(s)


def test_copy_on_write_keeps_the_source_intact(eng):
    e = eng
    a = e.open()
    e.prefill(a, prompt_rows(40, seed=11))
    before = kv_all(e, a, 40)
    b = e.fork(a, 40)
    fresh = e.open()
    try:
        other = prompt_rows(20, seed=12)
        e.reset(b)
        e.prefill(b, other)  # rewrites positions 0..19: pages shared with a are copied first
        e.prefill(fresh, other)
        after = kv_all(e, a, 40)
        for layer in range(12):
            assert np.array_equal(after[layer][0], before[layer][0])
            assert np.array_equal(after[layer][1], before[layer][1])
            kb, vb = e.kv(b, layer, 0, 20)
            kf, vf = e.kv(fresh, layer, 0, 20)
            assert np.array_equal(kb, kf) and np.array_equal(vb, vf)
    finally:
        for s in (a, b, fresh):
            e.close_stream(s)


def test_shared_pages_return_to_the_pool(pkg, weights_path):
    e = pkg.Engine(weights_path, device=0, max_streams=4, max_ctx=64, kv_pages=8)  # 8 pages of 16
    try:
        rows = prompt_rows(64, seed=21)
        a = e.open()
        e.prefill(a, rows)  # 4 pages
        b = e.fork(a, 64)   # shares all 4
        ref = kv_all(e, a, 64)
        e.close_stream(a)   # the pages stay alive for b
        got = kv_all(e, b, 64)
        for layer in range(12):
            assert np.array_equal(got[layer][0], ref[layer][0])
        c = e.open()
        e.prefill(c, rows)  # the other 4 pages
        with pytest.raises(pkg.MossGpuError, match="exhausted"):
            x = e.open()
            try:
                e.prefill(x, prompt_rows(16, seed=1))
            finally:
                e.close_stream(x)
        e.close_stream(b)
        e.close_stream(c)
        d, f = e.open(), e.open()
        e.prefill(d, rows)
        e.prefill(f, rows)  # all 8 pages again: nothing leaked
        e.close_stream(d)
        e.close_stream(f)
    finally:
        e.close()
