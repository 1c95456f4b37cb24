"""GPU parity of the fused attention kernel (bee_b200_attention) against the
oracle's per-head composition (scores, softmax, P.V in fp32 from the same
bf16-rounded inputs).  Tolerance (tests/_tol.py): bf16 output, the stated 1e-2
on the output's own scale (norm-wise 1e-2, element-wise 2e-2 of max(|O|, rms(O))), plus 1e-2 of
the per-element condition P.|V| of the final product."""
import ctypes

import numpy as np
import pytest

from tests._tol import assert_output_close, assert_scaled, attention_scale
from oracle.oracle import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _dev_bf16(torch, x):
    return torch.from_numpy(f32_to_bf16_bits(x).view(np.int16)).cuda()


def _run(torch, q, k, v, scale):
    from bee_b200 import _capi
    heads, seq, hd = q.shape
    dq, dk, dv = (_dev_bf16(torch, t) for t in (q, k, v))
    do = torch.empty(heads * seq * hd, dtype=torch.int16, device="cuda")
    _capi.call("bee_b200_attention", _capi.BF16, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(), heads,
               seq, hd, float(scale), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    code = ctypes.c_int(-1)
    _capi.call("bee_b200_device_status", ctypes.byref(code))
    assert code.value == 0, f"a pipeline wait gave up (code {code.value})"
    return bf16_bits_to_f32(do.cpu().numpy().view(np.uint16)).reshape(heads, seq, hd)


def _inputs(seed, heads, seq, hd, spread=1.0):
    rng = np.random.default_rng(seed)
    f = lambda: bf16_bits_to_f32(f32_to_bf16_bits((rng.standard_normal((heads, seq, hd)) * spread).astype(np.float32)))
    return f(), f(), f()


# odd tile counts (3 x 640: the last CTA of a head holds one tile) and longer rows
@pytest.mark.parametrize("heads,seq", [(1, 128), (2, 256), (3, 640), (1, 512), (2, 1024), (3, 1536)])
def test_attention_matches_oracle(cuda, oracle, heads, seq):
    torch = cuda
    q, k, v = _inputs(heads * 1000 + seq, heads, seq, 128)
    scale = float(1 / np.sqrt(128))
    got = _run(torch, q, k, v, scale)
    want = oracle.attention_f32(q, k, v, scale)
    assert_output_close(got, want, 1e-2, what=f"attention {heads}x{seq}", elementwise_rtol=2e-2)
    assert_scaled(got, want, attention_scale(q, k, v, scale), 1e-2, what=f"attention {heads}x{seq}")


def test_attention_large_scores_rescale(cuda, oracle):
    """Scores spread over a wide range (the running max keeps rising), which
    exercises the deferred rescale of the output accumulator."""
    torch = cuda
    heads, seq = 2, 512
    q, k, v = _inputs(7, heads, seq, 128, spread=1.0)
    # make later keys much larger so the max grows block after block
    k = k * np.linspace(0.5, 6.0, seq, dtype=np.float32)[None, :, None]
    k = bf16_bits_to_f32(f32_to_bf16_bits(k))
    scale = 0.25
    got = _run(torch, q, k, v, scale)
    want = oracle.attention_f32(q, k, v, scale)
    assert_output_close(got, want, 1e-2, what="attention rescale", elementwise_rtol=2e-2)
    assert_scaled(got, want, attention_scale(q, k, v, scale), 1e-2, what="attention rescale")


def test_attention_config_sampled_rows(cuda):
    """Config: Q, K, V [32, 2048, 128] N(0,1) bf16, scale 1/sqrt(128); rows of
    the output are independent, so 64 sampled query rows per head are checked
    against float64."""
    torch = cuda
    heads, seq, hd = 32, 2048, 128
    q, k, v = _inputs(2048, heads, seq, hd)
    scale = float(1 / np.sqrt(hd))
    got = _run(torch, q, k, v, scale)
    rows = np.random.default_rng(3).choice(seq, 64, replace=False)
    qs = q[:, rows].astype(np.float64)
    s = np.einsum("hid,hjd->hij", qs, k.astype(np.float64)) * scale
    s -= s.max(-1, keepdims=True)
    pm = np.exp(s)
    pm /= pm.sum(-1, keepdims=True)
    want = pm @ v.astype(np.float64)
    cond = pm @ np.abs(v.astype(np.float64))
    assert_output_close(got[:, rows], want, 1e-2, what="attention 32x2048x128 sampled rows", elementwise_rtol=2e-2)
    assert_scaled(got[:, rows], want, cond, 1e-2, what="attention config rows")


@pytest.mark.parametrize("heads,seq", [(2, 8192), (3, 4224)])
def test_attention_long_sequences_sampled_rows(cuda, heads, seq):
    """Long rows: 64 and 33 key blocks, so the two-stage K/V ring and the block
    pairs of the MMA loop go through many phases (and, at 4224 = 33 x 128, end on
    an odd block with an odd tile count); 48 sampled query rows per head against
    float64."""
    torch = cuda
    hd = 128
    q, k, v = _inputs(seq + heads, heads, seq, hd)
    scale = float(1 / np.sqrt(hd))
    got = _run(torch, q, k, v, scale)
    rows = np.unique(np.concatenate([np.random.default_rng(seq).choice(seq, 46, replace=False), [0, seq - 1]]))
    s_ = np.einsum("hid,hjd->hij", q[:, rows].astype(np.float64), k.astype(np.float64)) * scale
    s_ -= s_.max(-1, keepdims=True)
    pm = np.exp(s_)
    pm /= pm.sum(-1, keepdims=True)
    want = pm @ v.astype(np.float64)
    assert_output_close(got[:, rows], want, 1e-2, what=f"attention {heads}x{seq} sampled rows", elementwise_rtol=2e-2)


@pytest.mark.parametrize("heads,seq", [(20, 2048), (10, 4224), (150, 256), (37, 2048)])
def test_attention_persistent_schedules(cuda, heads, seq):
    """More units (a head's pair of query tiles) than SMs.  On a 148-SM B200,
    20 x 2048 (160 units, a last wave of 12) and 10 x 4224 (170 units of 33 key
    blocks, single-tile units among them) run as one persistent CTA per SM, each
    taking an equal share of the (unit, key block) sequence, so most shares end
    inside a unit and its two pieces are merged; 150 x 256 (units of two key
    blocks) and 37 x 2048 (two whole waves) keep one CTA per unit.  Three query
    rows in every 128-row tile (so every piece of every cut unit) against
    float64, and two calls must agree bit for bit (the merge does not depend on
    which piece finishes first)."""
    torch = cuda
    hd = 128
    q, k, v = _inputs(heads * 7 + seq, heads, seq, hd)
    scale = float(1 / np.sqrt(hd))
    got = _run(torch, q, k, v, scale)
    again = _run(torch, q, k, v, scale)
    assert np.array_equal(got, again), "two calls on the same inputs differ"
    rng = np.random.default_rng(seq + heads)
    rows = np.sort(np.concatenate([t * 128 + rng.choice(128, 3, replace=False) for t in range(seq // 128)]))
    s_ = np.einsum("hid,hjd->hij", q[:, rows].astype(np.float64), k.astype(np.float64)) * scale
    s_ -= s_.max(-1, keepdims=True)
    pm = np.exp(s_)
    pm /= pm.sum(-1, keepdims=True)
    want = pm @ v.astype(np.float64)
    assert_output_close(got[:, rows], want, 1e-2, what=f"attention {heads}x{seq} persistent", elementwise_rtol=2e-2)
    assert_scaled(got[:, rows], want, pm @ np.abs(v.astype(np.float64)), 1e-2, what=f"attention {heads}x{seq} persistent")


def test_attention_rejects_unsupported_shapes(cuda):
    from bee_b200 import _capi
    torch = cuda
    x = torch.empty(4 * 100 * 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_capi.BeeError, match="multiple"):
        _capi.call("bee_b200_attention", _capi.BF16, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 4, 100,
                   128, 0.1, None)
    with pytest.raises(_capi.BeeError, match="head_dim"):
        _capi.call("bee_b200_attention", _capi.BF16, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 128,
                   64, 0.1, None)
