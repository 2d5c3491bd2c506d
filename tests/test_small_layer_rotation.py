"""The residual-accumulator rotation of the two-launch layers (layer_small.cuh), modelled on the
CPU with the kernels' own index rules: launch p of a step (p = 2 * layer + half) reads x from
D[p % 3] (launch 0: the embedding rows), adds x + its output into D[(p + 1) % 3] (with integer
adds, in any order) and zeroes D[(p + 2) % 3], each for the step's rows r < R only.

Checked over random sequences of batch sizes (R changes from step to step, as decode batches
do): every launch adds into an accumulator whose rows r < R are zero, the step's result is in
D[0], D[1] is all zero again after every step, and the integer sums do not depend on the order
of the adds (the run-to-run determinism the fixed-point form is for)."""
from __future__ import annotations

import numpy as np

LAUNCHES = 24
HIDDEN = 16  # the model's 768 columns, shortened: the rule is per element
SCALE = 2.0 ** 32


def to_fixed(v):
    return np.rint(np.asarray(v, dtype=np.float64) * SCALE).astype(np.int64)


def run_step(D, x0, R, outputs, rng, shuffle=True):
    """One step of 24 launches; outputs[p] = the launch's contribution per row (float64).
    Returns the rows of D[0] after the step (the layers' result)."""
    for p in range(LAUNCHES):
        d_out, d_zero = D[(p + 1) % 3], D[(p + 2) % 3]
        assert not d_out[:R].any(), f"launch {p} adds into a non-zero accumulator"
        x = x0[:R] if p == 0 else D[p % 3][:R]
        x_fixed = to_fixed(x0[:R]) if p == 0 else x
        # the adds of one launch: x once (by the CTAs that also add the bias), then the
        # partial outputs of every CTA, in an order the hardware chooses
        parts = [x_fixed] + [to_fixed(outputs[p][:R] / 4)] * 4
        order = rng.permutation(len(parts)) if shuffle else range(len(parts))
        for i in order:
            d_out[:R] += parts[i]
        d_zero[:R] = 0
    return D[0][:R].copy()


def test_rotation_invariants_over_changing_batch_sizes():
    rng = np.random.default_rng(7)
    D = np.zeros((3, 8, HIDDEN), dtype=np.int64)  # the engine allocates the accumulators zeroed
    for step in range(40):
        R = int(rng.integers(1, 9))
        x0 = rng.standard_normal((8, HIDDEN))
        outputs = rng.standard_normal((LAUNCHES, 8, HIDDEN)) * 0.25
        res = run_step(D, x0, R, outputs, rng)
        assert not D[1].any(), f"step {step}: D[1] not zero after the step"
        # the result: x0 + the sum of every launch's output, to the fixed-point resolution
        want = x0[:R] + outputs[:, :R].sum(axis=0)
        assert np.abs(res / SCALE - want).max() < LAUNCHES * 5 / SCALE


def test_fixed_point_sums_do_not_depend_on_the_order_of_the_adds():
    rng = np.random.default_rng(11)
    x0 = rng.standard_normal((8, HIDDEN))
    outputs = rng.standard_normal((LAUNCHES, 8, HIDDEN))
    results = []
    for seed in range(4):
        D = np.zeros((3, 8, HIDDEN), dtype=np.int64)
        results.append(run_step(D, x0, 8, outputs, np.random.default_rng(seed)))
    for r in results[1:]:
        assert np.array_equal(r, results[0])
