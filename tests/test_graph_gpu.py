"""CUDA-graph replay of the forward (j1_model_launch captures a batch shape the second time it
is launched and replays it after that): every forward of a shape, direct, captured or
replayed, gives the same logits to the last bit; shapes interleave, a larger batch (which
reallocates the workspace and drops the graphs) does not disturb them, the per-launch
profiling pass and an injected launch failure run the kernels directly, and the kernel count
per forward is the same either way.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import julia1 as j1  # noqa: E402
from julia1 import synthetic  # noqa: E402


def _batch(lens, seed):
    rows = synthetic.synthetic_batch(lens, markers_per_seq=3, seed=seed, option_block=(4, 6, 8))
    return j1.Batch.new([j1.Encoded(*r) for r in rows])


@pytest.fixture(scope="module")
def model(torch_cuda):
    ck = synthetic.cached_checkpoint(seed=3, perturb=True)
    m = j1.CudaModel(ck, 0)
    yield m
    m.close()


def _forward(m, b):
    m.stage(b)
    m.launch()
    n = m.launch_count()
    return m.finish(int(b.marker_rows.size)), n


def test_replay_matches_direct_launches(model):
    a, b = _batch([300, 77, 512, 129], 1), _batch([64, 64, 1000], 2)
    ra, na = _forward(model, a)  # first sight of each shape: direct launches
    rb, nb = _forward(model, b)
    assert np.isfinite(ra).all() and np.isfinite(rb).all() and na > 0 and nb > 0
    for _ in range(3):  # second sight captures, then replays; the shapes interleave
        for bt, want, n_want in ((a, ra, na), (b, rb, nb)):
            got, n = _forward(model, bt)
            assert np.array_equal(got, want)
            assert n == n_want


def test_workspace_growth_drops_graphs(model):
    a = _batch([300, 77, 512, 129], 1)
    want, _ = _forward(model, a)
    _forward(model, a)
    big = _batch([1024] * 40, 4)  # more tokens than the workspace holds: it is reallocated
    rbig, _ = _forward(model, big)
    assert np.isfinite(rbig).all()
    for _ in range(3):
        got, _ = _forward(model, a)
        assert np.array_equal(got, want)
    assert np.array_equal(_forward(model, big)[0], rbig)


def test_profiling_and_injected_failures_launch_directly(model):
    a = _batch([200, 350, 90], 5)
    want, n = _forward(model, a)
    for _ in range(2):
        _forward(model, a)  # captured and replayed
    model.profile(True)
    try:
        got, n2 = _forward(model, a)
        fam = model.profile_read()
    finally:
        model.profile(False)
    assert np.array_equal(got, want) and n2 == n
    assert sum(v[1] for v in fam.values()) == n  # every kernel was launched (and timed) one by one
    j1.inject_fault(j1.FAULT_LAUNCH, 1)
    try:
        with pytest.raises(j1.J1Error, match="injected launch failure"):
            model.forward_flat(a)
    finally:
        j1.inject_fault(j1.FAULT_LAUNCH, 0)
    assert np.array_equal(_forward(model, a)[0], want)
