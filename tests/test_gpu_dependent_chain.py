"""Dependent ops back to back on one stream.  The streaming kernels (binary,
fp32->bf16 cast, row and global reduce, row softmax, the pipelined RMSNorm /
RoPE, the transposes, the broadcasting binary op) are launched so that the
next one may start while the previous one finishes, and each waits for its
predecessor before touching memory.  A chain in which every op reads the
previous op's output, and the next round overwrites buffers the previous
round read, must give bit for bit what the same chain gives with a device
synchronise after every op."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ADD, SUB, MUL, DIV = 0, 1, 2, 3
SUM, MAX = 0, 2


def _chain(torch, capi, x, y, xi, bufs, rounds, sync, rope):
    """Per round: a = x + y; b = a * y; c = b - a (reads both); h = bf16(c);
    r = rowsum(c); m = rowmax(b); s = softmax(c); z = rms_norm_rope(s, g);
    ht = transpose(h) (bf16); u = b - m (m broadcast along each row);
    w = xi + 1; t = int32 sum of w."""
    a, b, c, h, r, m, s, t, one, w, g, z, ht, u = bufs
    seq, heads, hd = rope
    I64 = ctypes.c_int64 * 2
    shape, full, bcast = I64(*x.shape), I64(x.shape[1], 1), I64(1, 0)
    st = torch.cuda.current_stream().cuda_stream
    rows, cols = x.shape
    n = x.numel()

    def op(name, *args):
        capi.call(name, *args)
        if sync:
            torch.cuda.synchronize()

    for _ in range(rounds):
        op("bee_b200_ew_binary", ADD, capi.F32, x.data_ptr(), y.data_ptr(), a.data_ptr(), n, st)
        op("bee_b200_ew_binary", MUL, capi.F32, a.data_ptr(), y.data_ptr(), b.data_ptr(), n, st)
        op("bee_b200_ew_binary", SUB, capi.F32, b.data_ptr(), a.data_ptr(), c.data_ptr(), n, st)
        op("bee_b200_ew_cast", capi.F32, c.data_ptr(), capi.BF16, h.data_ptr(), n, st)
        op("bee_b200_reduce_axis", SUM, capi.F32, c.data_ptr(), r.data_ptr(), rows, cols, 1, st)
        op("bee_b200_reduce_axis", MAX, capi.F32, b.data_ptr(), m.data_ptr(), rows, cols, 1, st)
        op("bee_b200_softmax_rows", capi.F32, c.data_ptr(), s.data_ptr(), rows, cols, st)
        op("bee_b200_rms_norm_rope", capi.F32, s.data_ptr(), g.data_ptr(), z.data_ptr(), rows, seq, heads, hd, 1e-6,
           10000.0, 0, st)
        op("bee_b200_transpose_2d", capi.BF16, h.data_ptr(), ht.data_ptr(), rows, cols, st)
        op("bee_b200_ew_binary_strided", SUB, capi.F32, 2, shape, b.data_ptr(), full, m.data_ptr(), bcast,
           u.data_ptr(), st)
        op("bee_b200_ew_binary", ADD, capi.I32, xi.data_ptr(), one.data_ptr(), w.data_ptr(), n, st)
        op("bee_b200_reduce_global", SUM, capi.I32, w.data_ptr(), t.data_ptr(), n, st)
    torch.cuda.synchronize()
    return [v.cpu().clone() for v in (a, b, c, h, r, m, s, t, w, z, ht, u)]


# RMSNorm+RoPE: 4096 = 32 heads x 128 (the pipelined kernel), 8200 = 41 heads x 200
# (an fp32 row above the pipe's 16 KiB: the plain kernel, launched without overlap)
@pytest.mark.parametrize("rows,cols,rope", [(4096, 4096, (64, 32, 128)), (333, 8200, (37, 41, 200))])
def test_dependent_chain_matches_synchronised_chain(cuda, rows, cols, rope):
    torch = cuda
    from bee_b200 import _capi
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = torch.randn(rows, cols, device="cuda", generator=g)
    y = torch.randn(rows, cols, device="cuda", generator=g)
    xi0 = torch.randint(-1000, 1001, (rows, cols), device="cuda", dtype=torch.int32, generator=g)
    one = torch.ones(rows, cols, device="cuda", dtype=torch.int32)
    gain = 1.0 + 0.02 * torch.randn(cols, device="cuda", generator=g)

    def fresh():
        return (torch.empty_like(x), torch.empty_like(x), torch.empty_like(x),
                torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16), torch.empty(rows, device="cuda"),
                torch.empty(rows, device="cuda"), torch.empty_like(x), torch.zeros(1, device="cuda", dtype=torch.int32),
                one, torch.empty_like(xi0), gain, torch.empty_like(x),
                torch.empty(cols, rows, device="cuda", dtype=torch.bfloat16), torch.empty_like(x))

    got = _chain(torch, _capi, x, y, xi0, fresh(), 20, sync=False, rope=rope)
    want = _chain(torch, _capi, x, y, xi0, fresh(), 20, sync=True, rope=rope)
    names = ["add", "mul", "sub", "cast", "row sum", "row max", "softmax", "int32 sum", "int32 add", "rms_norm_rope",
             "transpose", "b - rowmax"]
    for nm, g_, w_ in zip(names, got, want):
        assert torch.equal(g_, w_), f"{nm}: the back-to-back chain differs from the synchronised one"
    # and what the chain computes is right where it is exact
    xs, ys = x.cpu(), y.cpu()
    assert torch.equal(got[0], xs + ys) and torch.equal(got[1], (xs + ys) * ys)
    assert torch.equal(got[10], got[3].t()) and torch.equal(got[11], got[1] - got[5][:, None])
    w = xi0.cpu().numpy().astype(np.int64) + 1
    assert np.array_equal(got[8].numpy(), w.astype(np.int32))
    assert int(got[7].item()) == ((int(w.sum()) + 2**31) % 2**32) - 2**31


def test_attention_between_dependent_ops(cuda):
    """The fused attention also starts launching while the previous kernel on
    the stream finishes.  Here it reads an add's output and an add reads its
    output, back to back for five rounds (a bf16 add of zero copies exactly);
    the result must equal the chain synchronised after every op bit for bit."""
    torch = cuda
    from bee_b200 import _capi
    heads, seq = 6, 1024
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn(heads, seq, 128, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    zero = torch.zeros_like(q)
    n = q.numel()
    st = torch.cuda.current_stream().cuda_stream

    def run(sync):
        qq, o, o2 = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
        for r in range(5):
            src = q if r == 0 else o2
            _capi.call("bee_b200_ew_binary", ADD, _capi.BF16, src.data_ptr(), zero.data_ptr(), qq.data_ptr(), n, st)
            if sync:
                torch.cuda.synchronize()
            _capi.call("bee_b200_attention", _capi.BF16, qq.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), heads,
                       seq, 128, 0.088, st)
            if sync:
                torch.cuda.synchronize()
            _capi.call("bee_b200_ew_binary", ADD, _capi.BF16, o.data_ptr(), zero.data_ptr(), o2.data_ptr(), n, st)
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return o2.cpu()

    assert torch.equal(run(False), run(True)), "attention in a back-to-back chain differs from the synchronised chain"


def test_products_between_dependent_ops(cuda):
    """The single-CTA tensor-core GEMM and the kernels around it (fp32 matmul:
    split into bf16 pieces, products, partial sum; a 16-bit product with a
    small output and a long K: products of K chunks, then their sum) also
    launch early.  C1 = A . B (fp32), D = C1 + C1, C2 = D . B, and a bf16
    128 x 4096 x 4096 product of a cast of C2's rows, back to back for three
    rounds, must equal the chain synchronised after every op bit for bit."""
    torch = cuda
    from bee_b200 import _capi
    g = torch.Generator(device="cuda").manual_seed(21)
    n = 1024
    A = torch.rand(n, n, device="cuda", generator=g) * 2 - 1
    B = torch.rand(n, n, device="cuda", generator=g) * 2 - 1
    W = (torch.randn(4096, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream

    def run(sync):
        C1, D, C2 = (torch.empty(n, n, device="cuda") for _ in range(3))
        X = torch.empty(128, 4096, device="cuda", dtype=torch.bfloat16)
        Y = torch.empty(128, 4096, device="cuda", dtype=torch.bfloat16)

        def op(name, *args):
            _capi.call(name, *args)
            if sync:
                torch.cuda.synchronize()

        for _ in range(3):
            op("bee_b200_matmul", _capi.F32, A.data_ptr(), B.data_ptr(), C1.data_ptr(), n, n, n, st)
            op("bee_b200_ew_binary", ADD, _capi.F32, C1.data_ptr(), C1.data_ptr(), D.data_ptr(), n * n, st)
            op("bee_b200_matmul", _capi.F32, D.data_ptr(), B.data_ptr(), C2.data_ptr(), n, n, n, st)
            op("bee_b200_ew_cast", _capi.F32, C2.data_ptr(), _capi.BF16, X.data_ptr(), 128 * 4096, st)
            op("bee_b200_bmm", _capi.BF16, _capi.BF16, X.data_ptr(), W.data_ptr(), Y.data_ptr(), 1, 128, 4096, 4096, 0,
               1.0, st)
        torch.cuda.synchronize()
        return C1.cpu(), C2.cpu(), Y.cpu()

    for nm, a_, b_ in zip(["C1", "C2", "Y"], run(False), run(True)):
        assert torch.equal(a_, b_), f"{nm}: the back-to-back chain differs from the synchronised one"
