"""Parity of the forward at the other hidden widths the kernels support (256, 512, 1024,
and a one-layer head), against the oracle's BF16-chain restatement of the reference CUDA
path. Each width selects different GEMM instantiations (full-row units of 1, 2 or 4
sub-tiles of 256 columns; 4, 8 or 16 heads)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import julia1 as j1  # noqa: E402
from julia1 import synthetic  # noqa: E402
from oracle import oracle as orc  # noqa: E402

TOL_BF16 = 3e-2


@pytest.mark.parametrize("shape", [
    dict(hidden=256, heads=4, layers=3, intermediate=512, vocab=1000, max_positions=1024, head_layers=2),
    dict(hidden=512, heads=8, layers=3, intermediate=768, vocab=1000, max_positions=1024, head_layers=2),
    dict(hidden=1024, heads=16, layers=2, intermediate=1536, vocab=1000, max_positions=1024, head_layers=1),
], ids=["h256", "h512", "h1024"])
def test_width_parity(torch_cuda, tmp_path, shape):
    root = synthetic.write_checkpoint(str(tmp_path / "ck"), seed=3, perturb=True, **shape)
    rows = synthetic.synthetic_batch([700, 129, 1, 300], vocab=shape["vocab"], markers_per_seq=3, seed=150,
                                     mask_markers=False)
    b = j1.Batch.new([j1.Encoded(*r) for r in rows])
    m = j1.CudaModel(root, 0)
    try:
        gpu = m.forward_flat(b)
    finally:
        m.close()
    ref16 = orc.Oracle(root).forward_flat(b, mode="bf16")
    d = np.abs(gpu - ref16)
    print("h%d max|gpu-bf16| %.5f" % (shape["hidden"], d.max()))
    assert np.isfinite(gpu).all()
    assert d.max() <= TOL_BF16
