"""Prefill MUL_MAT with an F16 weight on the tcgen05 tensor cores
(b200_mul_mat_f16_tc), against the CPU oracle's ggml-cpu semantics
(src1 converted to f16, fp32 accumulation), column by column.

The reference keeps M >= 16 on CANN's own matmul over the ND copy
(patch:1200-1204); here every M > 8 runs on this kernel.  Shapes cover a
single partial tile (M = 9), the tile widths 64 / 128 / 256, several tiles
along M, rows and K that are not multiples of the 128 x 64 tile (TMA fills
the edges with zeros), and config 1's weight 8960 x 1536."""
import numpy as np
import pytest

import oracle as O
from helpers import TOL, assert_close, rng

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def B():
    import b200_decode

    return b200_decode


@pytest.mark.parametrize("n,k,m", [(256, 512, 9), (256, 512, 16), (384, 1024, 64), (200, 264, 130),
                                   (8960, 1536, 64), (8960, 1536, 512), (1024, 8192, 300)])
def test_mul_mat_f16_tc_matches_oracle(n, k, m):
    bw = B()
    r = rng(1000 + n + k + m)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    x = r.standard_normal((m, k)).astype(np.float32)
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(x).cuda()
    y = bw.mul_mat_f16_tc(dw, dx, n, k).cpu().numpy()
    assert y.shape == (m, n) and np.all(np.isfinite(y))
    for j in sorted({0, 1, m // 2, m - 1}):
        assert_close(y[j], O.mul_mat_f16(w, x[j]), TOL, f"column {j} of {m}")
    assert bw.device_status(reset=True) == 0


def test_mul_mat_f16_tc_strided_rows_and_routing():
    """x and y with row strides beyond k / n; mul_mat() of a packed F16
    weight routes M > 8 here and M <= 8 to the small-M kernel."""
    bw = B()
    r = rng(7)
    n, k, m = 512, 768, 40
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    x = r.standard_normal((m, k + 32)).astype(np.float32)
    dx = torch.from_numpy(x).cuda()[:, :k]
    y = torch.full((m, n + 16), float("nan"), device="cuda")[:, :n]
    bw.mul_mat_f16_tc(torch.from_numpy(w).cuda(), dx, n, k, y)
    yh = y.cpu().numpy()
    for j in (0, 17, m - 1):
        assert_close(yh[j], O.mul_mat_f16(w, x[j, :k]), TOL, f"strided column {j}")
    pw = bw.repack(bw.TYPE_F16, torch.from_numpy(w).cuda(), n, k)
    for mm in (4, 12):
        xx = torch.from_numpy(np.ascontiguousarray(x[:mm, :k])).cuda()
        out = bw.mul_mat(pw, xx).cpu().numpy()
        for j in range(mm):
            assert_close(out[j], O.mul_mat_f16(w, x[j, :k]), TOL, f"routed M={mm} column {j}")
    assert bw.device_status(reset=True) == 0
