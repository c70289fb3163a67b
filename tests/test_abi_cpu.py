"""CPU-side checks of the C ABI library: it loads, exports every entry point
that include/*.h declares, validates arguments before touching a device, and
its host helpers match the oracle."""
import glob
import os
import re

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(b200_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    import b200_decode as B

    L = B.lib()
    names = declared_symbols()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_version_and_errors():
    import b200_decode as B

    assert b"sm_100a" in B.lib().b200_version()
    assert B.lib().b200_strerror(-1) == b"invalid argument"


@pytest.mark.parametrize("wtype,n,k", [(1, 8960, 1536), (2, 1536, 8960), (8, 151936, 1536), (2, 10240, 8192),
                                       (2, 57344, 8192), (2, 8192, 28672), (1, 5, 8), (8, 3, 32)])
def test_packed_size_layout(wtype, n, k):
    import b200_decode as B

    u = k // 8 if wtype == 1 else k // 32
    pad16 = lambda v: (v + 15) // 16 * 16
    rs = {1: 2 * k, 2: 16 * u + pad16(2 * u), 8: 32 * u + pad16(2 * u)}[wtype]
    assert B.row_stride(wtype, n, k) == rs
    assert B.packed_size(wtype, n, k) == rs * n
    assert rs % 16 == 0


@pytest.mark.parametrize("n,k", [(151936, 1536), (8960, 1536), (3, 32), (5, 96)])
def test_packed_size_a8w8(n, k):
    import b200_decode as B

    # int8 rows of k bytes, then the n f16 row scales padded to 16 bytes
    pad16 = lambda v: (v + 15) // 16 * 16
    assert B.row_stride(B.TYPE_A8W8, n, k) == k
    assert B.packed_size(B.TYPE_A8W8, n, k) == n * k + pad16(2 * n)


def test_unsupported_shapes_report_zero():
    import b200_decode as B

    assert B.packed_size(2, 16, 48) == 0      # K not a multiple of 32
    assert B.packed_size(1, 16, 12) == 0      # F16 K not a multiple of 8
    assert B.packed_size(3, 16, 64) == 0      # type not served


def test_argument_validation_without_device():
    import ctypes as C

    import b200_decode as B

    L = B.lib()
    assert L.b200_gemv_f16(None, None, None, 8, 8, None) == B.EINVAL
    assert L.b200_fa_decode(None, None, None, None, None, None, 128, 12, 2, 16, 0, 0, 0, 0, 1.0, None, 0,
                            None) == B.EINVAL
    assert L.b200_fa_workspace_size(128, 12, 5, 16) == 0
    assert L.b200_repack(2, None, None, 4, 64, None) == B.EINVAL
    assert L.b200_quantize_q8_0(None, None, 32, None) == B.EINVAL
    v = C.c_uint(0)
    assert L.b200_device_status(None, 0) == B.EINVAL
    # neighbour ops: null pointers and bad shapes are refused before any launch
    assert L.b200_rms_norm_f32(None, None, None, 8, 1, 1e-5, None) == B.EINVAL
    assert L.b200_rope_norm_f32(None, None, None, 1, 8, 127, 1e4, None) == B.EINVAL
    assert L.b200_set_rows_f16(None, None, None, 8, 1, 16, 4, None) == B.EINVAL
    assert L.b200_get_rows_q4_0(None, None, None, 48, 1, 4, None) == B.EINVAL
    assert L.b200_swiglu_f32(None, None, None, 8, None) == B.EINVAL
    assert L.b200_add_f32(None, None, None, 8, None) == B.EINVAL
    assert L.b200_argmax_f32(None, 8, None, None) == B.EINVAL
    assert L.b200_get_rows_q4_0_packed(None, None, None, 64, 1, 4, None) == B.EINVAL
    h = C.c_void_p()
    assert L.b200_upload_begin(2, 4, 64, None, C.byref(h)) == B.EINVAL
    assert L.b200_upload_write(None, 0, None, 16, None) == B.EINVAL
    assert L.b200_upload_end(None) == B.EINVAL
    assert L.b200_mul_mat_f16(None, None, None, 16, 64, 2, 64, 16, None) == B.EINVAL
    fake = C.c_void_p(256)  # never dereferenced: each call fails validation first
    assert L.b200_mul_mat_f16(fake, fake, fake, 16, 64, 9, 64, 16, None) == B.EINVAL   # m > 8
    assert L.b200_mul_mat_f16(fake, fake, fake, 16, 60, 2, 64, 16, None) == B.EINVAL   # k % 8
    assert L.b200_mul_mat_f16(fake, fake, fake, 16, 64, 2, 32, 16, None) == B.EINVAL   # ldx < k
    assert L.b200_a8w8_transform(None, None, 4, 64, None) == B.EINVAL
    assert L.b200_gemv_a8w8(None, None, None, 4, 64, None) == B.EINVAL


def test_kv_lengths_host_helper_matches_oracle():
    import b200_decode as B

    r = np.random.default_rng(0)
    m = np.zeros((6, 300), np.float16)
    for i, cut in enumerate([300, 1, 0, 150, 299, 7]):
        m[i, cut:] = -np.inf
    m[3, 20] = -np.inf  # interior -inf does not shorten the row
    np.testing.assert_array_equal(B.kv_lengths_from_mask(m), O.kv_lengths_from_mask(m))
    np.testing.assert_array_equal(B.kv_lengths_from_mask(m), [300, 1, 1, 150, 299, 7])


@pytest.mark.parametrize("name,wtype,ne,disable,tied,want", [
    ("blk.0.ffn_gate.weight", 1, (1536, 8960, 1, 1), None, False, True),
    ("blk.11.ffn_up.weight", 1, (1536, 8960, 1, 1), "", False, True),
    ("blk.11.ffn_down.weight", 1, (8960, 1536, 1, 1), "11", False, False),
    ("blk.11.ffn_down.weight", 1, (8960, 1536, 1, 1), "0-3, 10-12", False, False),
    ("blk.4.ffn_down.weight", 1, (8960, 1536, 1, 1), "0-3, 10-12", False, True),
    ("blk.3.ffn_up.weight", 1, (1536, 8960, 1, 1), ",, 3 ,", False, False),
    ("blk.3.attn_q.weight", 1, (1536, 1536, 1, 1), None, False, False),        # not an FFN weight
    ("blk.3.ffn_up.weight", 2, (1536, 8960, 1, 1), None, False, False),        # Q4_0: not F16
    ("blk.3.ffn_up.weight", 1, (1536, 8960, 2, 1), None, False, False),        # batched
    ("ffn_up.weight", 1, (1536, 8960, 1, 1), "0-99", False, True),             # no layer number
    ("token_embd.weight", 1, (1536, 151936, 1, 1), None, True, True),
    ("token_embd.weight", 1, (1536, 151936, 1, 1), None, False, False),
    ("token_embd.weight", 1, (896, 151936, 1, 1), None, True, False),          # other shape
])
def test_a8w8_weight_policy(name, wtype, ne, disable, tied, want):
    """ggml_cann_310b_is_a8w8_weight / _layer_disabled (patch:1481-1533)."""
    import b200_decode as B

    assert B.a8w8_selects_weight(name, wtype, ne, disable, tied) is want


@pytest.mark.parametrize("bad", ["x", "3-", "-3", "1,a-4"])
def test_a8w8_weight_policy_malformed_list(bad):
    import b200_decode as B

    with pytest.raises(B.B200Error):
        B.a8w8_selects_weight("blk.5.ffn_up.weight", 1, (1536, 8960, 1, 1), bad)


def test_gemv_uneven_cta_shares(tmp_path):
    """gemv_cta_start (csrc/args.h), the row split of a GEMV whose last CTAs
    start late: compiled on the host and checked to cover [0, items) in
    order with every CTA's share, the late CTAs' share near pct % of the
    others', and the even split whenever the skew is off."""
    import shutil
    import subprocess

    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no g++")
    src = tmp_path / "split.cpp"
    src.write_text(r'''
#include <cstdio>
#include "args.h"
using b200::gemv_cta_start;
int main() {
    const long cases[][4] = {{148, 8192, 64, 65}, {148, 8192, 64, 100}, {148, 28672, 16, 50}, {148, 4096, 0, 65},
                             {132, 5120, 131, 65}, {148, 200, 64, 30}};
    for (auto& c : cases) {
        const long grid = c[0], items = c[1], late = c[2], pct = c[3];
        long prev = gemv_cta_start(0, grid, items, late, pct);
        if (prev != 0) return 1;
        long early_max = 0, late_min = items;
        for (long i = 0; i < grid; ++i) {
            const long a = gemv_cta_start(i, grid, items, late, pct), b = gemv_cta_start(i + 1, grid, items, late, pct);
            if (b < a) return 2;
            if (late == 0 || pct >= 100) {
                if (a != i * items / grid) return 3;
            }
            if (i < grid - late) early_max = b - a > early_max ? b - a : early_max;
            else late_min = b - a < late_min ? b - a : late_min;
        }
        if (gemv_cta_start(grid, grid, items, late, pct) != items) return 4;
        printf("%ld %ld %ld %ld %ld %ld\n", grid, items, late, pct, early_max, late_min);
    }
    return 0;
}
''')
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = tmp_path / "split"
    inc = [f"-I{os.path.join(root, 'llama-cpp-ascend310b4-addon_b200', 'csrc')}", "-I/usr/local/cuda/include"]
    r = subprocess.run([gxx, "-std=c++17", "-O1", *inc, str(src), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stdout)
    for ln in r.stdout.split("\n"):
        if not ln:
            continue
        grid, items, late, pct, early_max, late_min = map(int, ln.split())
        if 0 < late < grid and pct < 100 and items >= 4 * grid:
            # the late CTAs' share is pct % of the early ones' (to a row)
            assert abs(late_min - early_max * pct / 100) <= 2, ln
