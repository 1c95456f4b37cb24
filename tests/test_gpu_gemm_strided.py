"""GPU parity of bee_b200_bmm_strided (batched products over strided views)
against the oracle's bf16 / fp32 GEMM on the materialised views.  Tolerances as
tests/test_gpu_gemm.py: bf16 outputs 1e-2, fp32 outputs 1e-4 of the |A||B|
condition.  Every case also checks that nothing outside the C view changed."""
import ctypes

import numpy as np
import pytest

from tests._tol import assert_dot_close
from oracle.oracle import Oracle, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu
SENTINEL = 0x7FC1  # a bf16 NaN pattern no product produces


def run_strided(torch, dt_in, dt_out, a_buf, a_off, lda, sa, b_buf, b_off, ldb, sb, c_len, c_off, ldc, sc, batch, m,
                k, n, b_trans, alpha=1.0, c_byte_shift=0):
    from bee_b200 import _capi
    as_t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).cuda()
    da, db = as_t(a_buf), as_t(b_buf)
    out_np = np.uint16 if dt_out == _capi.BF16 else np.float32
    es_out = np.dtype(out_np).itemsize
    init = np.full(c_len + 8, SENTINEL if dt_out == _capi.BF16 else np.nan, dtype=out_np)
    dc = torch.from_numpy(init.view(np.int16) if out_np == np.uint16 else init).cuda()
    es_in = a_buf.dtype.itemsize
    _capi.call("bee_b200_bmm_strided", dt_in, dt_out, da.data_ptr() + a_off * es_in, lda, sa,
               db.data_ptr() + b_off * es_in, ldb, sb, dc.data_ptr() + c_off * es_out + c_byte_shift, ldc, sc,
               batch, m, k, n, b_trans, alpha, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    c = dc.cpu().numpy()
    return c.view(np.uint16) if out_np == np.uint16 else c


def views(a_buf, a_off, lda, sa, b_buf, b_off, ldb, sb, batch, m, k, n, b_trans):
    a = Oracle.strided_gather(a_buf, a_off, (batch, m, k), (sa, lda, 1))
    if b_trans:
        b = Oracle.strided_gather(b_buf, b_off, (batch, n, k), (sb, ldb, 1)).transpose(0, 2, 1)
    else:
        b = Oracle.strided_gather(b_buf, b_off, (batch, k, n), (sb, ldb, 1))
    return a, np.ascontiguousarray(b)


def check_c(c, c_off, ldc, sc, batch, m, n, want, a32, b32, out_bf16, tol):
    idx = Oracle.strided_gather(np.arange(c.size, dtype=np.int64), c_off, (batch, m, n), (sc, ldc, 1))
    got = c[idx]
    got32 = bf16_bits_to_f32(got) if out_bf16 else got
    for bb in range(batch):
        assert_dot_close(got32[bb], want[bb], a32[bb], b32[bb], tol, what=f"batch {bb}")
    outside = np.ones(c.size, bool)
    outside[idx.reshape(-1)] = False
    rest = c[outside]
    if out_bf16:
        assert np.all(rest == SENTINEL), "a write landed outside the C view"
    else:
        assert np.all(np.isnan(rest)), "a write landed outside the C view"


CASES = [
    # batch, m, k, n, lda_pad, ldb_pad, ldc_pad, batch pads, b_trans
    (3, 300, 264, 520, 24, 8, 40, (64, 16, 8), 0),
    (2, 257, 128, 129, 8, 0, 3, (8, 0, 5), 1),
    (1, 64, 96, 72, 32, 16, 8, (0, 0, 0), 0),
    (4, 128, 256, 256, 0, 0, 0, (0, 0, 0), 1),
]


@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_bmm_strided_bf16(cuda, oracle, out, case):
    from bee_b200 import _capi
    batch, m, k, n, pa, pb, pc, (xa, xb, xc), bt = case
    lda, ldb, ldc = k + pa, (k if bt else n) + pb, n + pc
    sa, sb, sc = m * lda + xa, (n if bt else k) * ldb + xb, m * ldc + xc
    rng = np.random.default_rng(batch * 1000 + m + n)
    a_buf = f32_to_bf16_bits(rng.standard_normal(batch * sa + 16).astype(np.float32))
    b_buf = f32_to_bf16_bits(rng.standard_normal(batch * sb + 16).astype(np.float32))
    a_off, b_off, c_off = 8, 16, 8
    a, b = views(a_buf, a_off, lda, sa, b_buf, b_off, ldb, sb, batch, m, k, n, bt)
    want = oracle.bmm_bf16(a, b)
    c = run_strided(cuda, _capi.BF16, _capi.BF16 if out == "bf16" else _capi.F32, a_buf, a_off, lda, sa, b_buf, b_off,
                    ldb, sb, batch * sc + 16, c_off, ldc, sc, batch, m, k, n, bt)
    check_c(c, c_off, ldc, sc, batch, m, n, want, bf16_bits_to_f32(a), bf16_bits_to_f32(b), out == "bf16",
            1e-2 if out == "bf16" else 1e-4)


@pytest.mark.parametrize("contiguous_a", [True, False])
def test_bmm_strided_shared_b(cuda, oracle, contiguous_a):
    """stride_b = 0: one B for every batch (stacked into one product when A and C
    batches are contiguous, else the SIMT kernel)."""
    from bee_b200 import _capi
    batch, m, k, n = 3, 200, 128, 264
    lda = k if contiguous_a else k + 8
    sa, ldb, ldc = m * lda, n, n
    sc = m * ldc
    rng = np.random.default_rng(17)
    a_buf = f32_to_bf16_bits(rng.standard_normal(batch * sa).astype(np.float32))
    b_buf = f32_to_bf16_bits(rng.standard_normal(k * n).astype(np.float32))
    a, b = views(a_buf, 0, lda, sa, b_buf, 0, ldb, 0, batch, m, k, n, 0)
    want = oracle.bmm_bf16(a, b)
    c = run_strided(cuda, _capi.BF16, _capi.F32, a_buf, 0, lda, sa, b_buf, 0, ldb, 0, batch * sc, 0, ldc, sc, batch, m,
                    k, n, 0)
    check_c(c, 0, ldc, sc, batch, m, n, want, bf16_bits_to_f32(a), bf16_bits_to_f32(b), False, 1e-4)


def test_bmm_strided_unaligned_falls_back(cuda, oracle):
    """lda not a multiple of 8 and a C pointer off the 16-byte grid: SIMT path and
    element stores, same results."""
    from bee_b200 import _capi
    batch, m, k, n = 2, 150, 100, 140
    lda, ldb, ldc = k + 3, n, n + 1
    sa, sb, sc = m * lda, k * ldb, m * ldc
    rng = np.random.default_rng(23)
    a_buf = f32_to_bf16_bits(rng.standard_normal(batch * sa).astype(np.float32))
    b_buf = f32_to_bf16_bits(rng.standard_normal(batch * sb).astype(np.float32))
    a, b = views(a_buf, 0, lda, sa, b_buf, 0, ldb, sb, batch, m, k, n, 0)
    want = oracle.bmm_bf16(a, b)
    c = run_strided(cuda, _capi.BF16, _capi.BF16, a_buf, 0, lda, sa, b_buf, 0, ldb, sb, batch * sc + 8, 1, ldc, sc,
                    batch, m, k, n, 0)
    check_c(c, 1, ldc, sc, batch, m, n, want, bf16_bits_to_f32(a), bf16_bits_to_f32(b), True, 1e-2)


def test_bmm_strided_f32_and_k0(cuda, oracle):
    from bee_b200 import _capi
    batch, m, k, n = 2, 33, 17, 45
    lda, ldb, ldc = 20, 50, 47
    sa, sb, sc = m * lda + 1, k * ldb + 2, m * ldc + 3
    rng = np.random.default_rng(29)
    a_buf = rng.standard_normal(batch * sa).astype(np.float32)
    b_buf = rng.standard_normal(batch * sb).astype(np.float32)
    a, b = views(a_buf, 0, lda, sa, b_buf, 0, ldb, sb, batch, m, k, n, 0)
    want = np.stack([oracle.matmul_f32(a[i], b[i]) for i in range(batch)])
    c = run_strided(cuda, _capi.F32, _capi.F32, a_buf, 0, lda, sa, b_buf, 0, ldb, sb, batch * sc, 0, ldc, sc, batch,
                    m, k, n, 0)
    check_c(c, 0, ldc, sc, batch, m, n, want, a, b, False, 1e-5)
    # K = 0: C = 0 inside the view
    c0 = run_strided(cuda, _capi.F32, _capi.F32, a_buf, 0, lda, sa, b_buf, 0, ldb, sb, batch * sc, 0, ldc, sc, batch,
                     m, 0, n, 0)
    idx = Oracle.strided_gather(np.arange(c0.size, dtype=np.int64), 0, (batch, m, n), (sc, ldc, 1))
    assert np.all(c0[idx] == 0)


def test_bmm_strided_rejects_bad_views(cuda):
    from bee_b200 import _capi
    st = None
    with pytest.raises(_capi.BeeError, match="leading dimension"):
        _capi.call("bee_b200_bmm_strided", 4, 4, 16, 3, 12, 16, 4, 16, 16, 4, 16, 1, 4, 4, 4, 0, 1.0, st)
    with pytest.raises(_capi.BeeError, match="overlap"):
        _capi.call("bee_b200_bmm_strided", 4, 4, 16, 4, 16, 16, 4, 16, 16, 4, 8, 2, 4, 4, 4, 0, 1.0, st)
