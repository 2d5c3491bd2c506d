"""Batched prefill (several streams' prompts in shared passes through the layers) and the
direct tensor-core GEMM form it runs on (one CTA per 128 weight rows x <= 256 batch rows,
every K chunk, accumulators read straight from TMEM), against the C oracle's A16 prefill
(LlmModel::prefill, llm.cpp:327-401, one stream at a time).  Same tolerances as
test_gpu_parity.py."""
from __future__ import annotations

import numpy as np
import pytest

from golden_inputs import forced_codes, fp16_normal, global_state, prompt_rows
from oracle_py import Oracle, sample_params
from test_gpu_parity import KL_TOL, TOL, kl_per_frame

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pkg():
    import moss_b200
    moss_b200.build()
    return moss_b200


_ORACLE = {}


def oracle_prompt(weights_path, L, seed):
    """The oracle after prefilling prompt_rows(L, seed), computed once per module."""
    if (L, seed) not in _ORACLE:
        _ORACLE[(L, seed)] = oracle_prefilled(weights_path, rows=prompt_rows(L, seed=seed))
    return _ORACLE[(L, seed)]


def oracle_prefilled(weights_path, rows=None, x=None, start_rows=None):
    o = Oracle(weights_path, max_ctx=1100, a16_prefill=True)
    if start_rows is not None:
        o.prefill_rows(start_rows)
    if rows is not None:
        o.prefill_rows(rows, start=o.position)
    else:
        o.prefill_embeds(x, start=o.position)
    return o


def check_stream(e, sid, o, n_pos):
    assert e.position(sid) == o.position == n_pos
    assert np.abs(e.hidden(sid) - o.hidden()).max() < TOL
    for layer in (0, 6, 11):
        pick = sorted({0, n_pos // 2, n_pos - 1})
        kk, vv = e.kv(sid, layer, 0, n_pos)
        ok, ov = o.kv(layer, 0, n_pos)
        assert np.abs(kk[pick] - ok[pick]).max() < TOL
        assert np.abs(vv[pick] - ov[pick]).max() < TOL


@pytest.mark.parametrize("max_rows,direct", [(1024, 16), (64, 16), (1024, 0), (256, 128)])
def test_prefill_batch_matches_per_stream_oracle(pkg, weights_path, max_rows, direct):
    # direct = 16: every GEMM of the passes in the direct form (one 160-row slice, or 64-row
    # passes); direct = 0: split-K clusters throughout; (256, 128): a 160-row direct slice.
    # max_rows = 64: streams span several passes.
    lens = [24, 70, 7, 57]
    e = pkg.Engine(weights_path, device=0, max_streams=8, max_ctx=1100, max_rows=max_rows)
    try:
        e.set_tc_policy(direct, 256)
        prompts = [prompt_rows(L, seed=100 + i) for i, L in enumerate(lens)]
        sids = [e.open() for _ in lens]
        e.prefill_batch(sids, prompts)
        for i in (0, 1, 2, 3):
            check_stream(e, sids[i], oracle_prompt(weights_path, lens[i], 100 + i), lens[i])
    finally:
        e.close()


def test_prefill_embeds_batch_continues_existing_prefixes(pkg, weights_path):
    # starts > 0: each stream already holds a prefix; the batch appends to it
    e = pkg.Engine(weights_path, device=0, max_streams=4, max_ctx=1100, max_rows=512)
    try:
        e.set_tc_policy(16, 128)
        rng = np.random.default_rng(9)
        heads = [prompt_rows(L, seed=200 + i) for i, L in enumerate((10, 17))]
        xs = [fp16_normal(rng, (L, 768)) for L in (40, 21)]
        sids = [e.open(), e.open()]
        for s, h in zip(sids, heads):
            e.prefill(s, h)
        e.prefill_embeds_batch(sids, xs, starts=[10, 17])
        for i, s in enumerate(sids):
            o = oracle_prefilled(weights_path, x=xs[i], start_rows=heads[i])
            check_stream(e, s, o, len(heads[i]) + len(xs[i]))
    finally:
        e.close()


def test_direct_form_decode_frames_match_oracle(pkg, weights_path):
    # a decode batch forced onto the direct GEMM form (slices of 16..64 rows): teacher-forced
    # frames against the oracle, and the same frames through the split-K form
    lens = [33, 64, 100, 129, 17, 250, 48, 90, 5, 300, 61, 77, 160, 15, 44, 200, 31, 99, 8, 140]
    e = pkg.Engine(weights_path, device=0, max_streams=len(lens) + 1, max_ctx=1100)
    try:
        out = {}
        for direct in (16, 0):
            e.set_tc_policy(direct, 64)
            sids = [e.open() for _ in lens]
            states = [global_state(L, seed=300 + i) for i, L in enumerate(lens)]
            for s, (k, v, h0, _) in zip(sids, states):
                e.set_state(s, k, v, h0)
                e.generate_begin(s, 0)
            p = pkg.SampleParams.make(greedy=True, repetition_penalty=1.2, min_frames=99)
            forced = forced_codes(len(lens), seed=31)
            _, _, _, logits = e.step(sids, p, forced=forced, want_logits=True)
            out[direct] = (logits, np.stack([e.hidden(s) for s in sids]))
            if direct:
                for i in (0, 5, 9, 13):
                    k, v, h0, _ = states[i]
                    o = Oracle(weights_path, max_ctx=1100)
                    o.set_state(k, v, h0)
                    oc, ol, _ = o.generate(2, sample_params(greedy=True, rep=1.2, min_frames=99),
                                           forced=np.stack([forced[i], forced[i]]), want_logits=True)
                    assert np.abs(logits[i] - ol[0]).max() <= TOL
                    assert kl_per_frame(ol[:1], logits[i][None]).max() <= KL_TOL
                    assert np.abs(e.hidden(sids[i]) - o.hidden()).max() < TOL
            for s in sids:
                e.close_stream(s)
        assert np.abs(out[16][0] - out[0][0]).max() <= TOL
        assert np.abs(out[16][1] - out[0][1]).max() <= TOL
    finally:
        e.close()


def test_prefill_batch_rejects_bad_batches(pkg, weights_path):
    e = pkg.Engine(weights_path, device=0, max_streams=4, max_ctx=256)
    try:
        a, b = e.open(), e.open()
        with pytest.raises(pkg.MossGpuError, match="repeated"):
            e.prefill_batch([a, a], [prompt_rows(4, seed=1), prompt_rows(4, seed=2)])
        with pytest.raises(pkg.MossGpuError, match="not open"):
            e.prefill_batch([a, 3], [prompt_rows(4, seed=1), prompt_rows(4, seed=2)])
        bad = prompt_rows(4, seed=1)
        bad[2, 0] = 16384
        with pytest.raises(pkg.MossGpuError, match="text id"):
            e.prefill_batch([a, b], [prompt_rows(4, seed=1), bad])
        assert e.position(a) == 0 and e.position(b) == 0
    finally:
        e.close()


def test_prefill_batch_after_long_prefixes_merges_chunks(pkg, weights_path):
    # prefixes of 600 and 1030 positions: the new rows' groups attend over 2 and 3 chunks
    # (partials per chunk, merged by the combine kernel); 13 and 9 rows make partial groups
    e = pkg.Engine(weights_path, device=0, max_streams=4, max_ctx=1100, max_rows=64)
    try:
        e.set_tc_policy(16, 64)
        plan = [(600, 13, 51), (1030, 9, 52)]
        sids, states, rows = [], [], []
        for L, n, seed in plan:
            s = e.open()
            k, v, h0, _ = global_state(L, seed=seed)
            e.set_state(s, k, v, h0)
            sids.append(s)
            states.append((k, v, h0))
            rows.append(prompt_rows(n, seed=seed + 10))
        e.prefill_batch(sids, rows, starts=[L for L, _, _ in plan])
        for i, (L, n, _) in enumerate(plan):
            k, v, h0 = states[i]
            o = Oracle(weights_path, max_ctx=1100, a16_prefill=True)
            o.set_state(k, v, h0)
            o.prefill_rows(rows[i], start=L)
            assert e.position(sids[i]) == o.position == L + n
            assert np.abs(e.hidden(sids[i]) - o.hidden()).max() < TOL
            for layer in (0, 11):
                kk, vv = e.kv(sids[i], layer, L, n)
                ok, ov = o.kv(layer, L, n)
                assert np.abs(kk - ok).max() < TOL
                assert np.abs(vv - ov).max() < TOL
    finally:
        e.close()
