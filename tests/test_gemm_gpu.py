# SPDX-License-Identifier: MIT
"""GPU: the tensor-core matmul (tcgen05 kind::i8, include/qh_backend.h
qh_gemm*) against the oracle's restatement of tensor_matmul_*_f32
(slm/tensor.c:827-1033) on the same seeded inputs. Bar: bit-exact fp32 --
the integers come from the tensor core, the per-block fp32 combination
follows the reference's order."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_bitwise(got, want, what):
    if not np.array_equal(bits(got), bits(want)):
        bad = np.flatnonzero(bits(got).ravel() != bits(want).ravel())
        i = bad[0]
        raise AssertionError(f"{what}: {bad.size} of {got.size} differ, first at {np.unravel_index(i, got.shape)}: "
                             f"got {got.ravel()[i]!r} want {want.ravel()[i]!r}")


def run_gemm(qh, cuda, gt, w_np, k, out_f, x_np):
    w = qh.host.to_device(w_np)
    x = qh.host.to_device(np.ascontiguousarray(x_np, np.float32))
    out = qh.host.matmul_gemm(gt, w, k, out_f, x, n_tok=x_np.shape[0])
    cuda.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("gt", [Q4_K, Q5_K, Q6_K])
@pytest.mark.parametrize("k,out_f,n_tok", [(256, 128, 64), (1024, 300, 70), (2048, 257, 1), (512, 1000, 129)])
def test_gemm_bitexact_vs_oracle(qh, cuda, oracle, gt, k, out_f, n_tok):
    w = qh.host.synth_blocks(gt, out_f * (k // 256), 0x6E44 + gt + k + out_f)
    x = qh.host.synth_normal(n_tok * k, 77 + n_tok + k, 0.0, 1.0).reshape(n_tok, k)
    got = run_gemm(qh, cuda, gt, w, k, out_f, x)
    want = oracle.matmul(gt, w, out_f, k, x)
    assert_bitwise(got, want.reshape(n_tok, out_f), f"type {gt} k={k} out_f={out_f} n={n_tok}")


def test_gemm_matches_gemv_path(qh, cuda):
    """Same inputs through the matvec kernel (qh_matmul) and the GEMM."""
    k, out_f, n_tok = 1024, 2048, 96
    w_np = qh.host.synth_blocks(Q4_K, out_f * 4, 0xA11)
    x_np = qh.host.synth_normal(n_tok * k, 0xA12).reshape(n_tok, k)
    w, x = qh.host.to_device(w_np), qh.host.to_device(x_np)
    a = qh.host.matmul(Q4_K, w, k, out_f, x, n_tok=n_tok)
    b = qh.host.matmul_gemm(Q4_K, w, k, out_f, x, n_tok=n_tok)
    cuda.cuda.synchronize()
    assert_bitwise(b.cpu().numpy(), a.cpu().numpy(), "gemm vs gemv")


def test_grouped_gemm_with_row_stride(qh, cuda, oracle):
    """Two jobs sharing one tiled activation buffer; outputs with ld_out > out_f."""
    torch = cuda
    k, n_tok = 1024, 65
    shapes = [(384, Q6_K), (200, Q6_K)]
    x_np = qh.host.synth_normal(n_tok * k, 5).reshape(n_tok, k)
    xq = qh.host.quantize_q8kt(qh.host.to_device(x_np), k, n_tok)
    jobs, ws, outs = [], [], []
    for i, (out_f, gt) in enumerate(shapes):
        w = qh.host.synth_blocks(gt, out_f * 4, 900 + i)
        ws.append(w)
        wt = qh.host.gemm_pack(gt, qh.host.to_device(w), k, out_f)
        out = torch.full((n_tok, out_f + 13), -7.0, dtype=torch.float32, device="cuda")
        outs.append((wt, out))
        jobs.append((wt, out_f, out, out_f + 13))
    qh.host.gemm(Q6_K, jobs, k, xq, n_tok)
    cuda.cuda.synchronize()
    for (out_f, gt), w, (_, out) in zip(shapes, ws, outs):
        o = out.cpu().numpy()
        assert_bitwise(o[:, :out_f], oracle.matmul(gt, w, out_f, k, x_np).reshape(n_tok, out_f), f"job {out_f}")
        assert np.all(o[:, out_f:] == -7.0), "wrote past out_f"


@pytest.mark.parametrize("gt,k,out_f,n_tok", [(Q6_K, 3584, 1024, 64), (Q4_K, 2048, 1024, 64),
                                               (Q5_K, 1024, 300, 130), (Q4_K, 256, 128, 1)])
def test_split_k_equals_unsplit(qh, cuda, oracle, gt, k, out_f, n_tok):
    """Few output tiles: the super-blocks are split over CTAs and the terms
    added in block order by the last one -- bit-identical to one CTA per tile
    and to the oracle. Run twice on one scratch (counters must return to 0)."""
    w = qh.host.synth_blocks(gt, out_f * (k // 256), 0x5B + k + gt)
    x_np = qh.host.synth_normal(n_tok * k, 0x5C + k).reshape(n_tok, k)
    wt = qh.host.gemm_pack(gt, qh.host.to_device(w), k, out_f)
    xq = qh.host.quantize_q8kt(qh.host.to_device(x_np), k, n_tok)
    outs = []
    for split in (False, True):
        out = cuda.empty((n_tok, out_f), dtype=cuda.float32, device="cuda")
        scratch = qh.host.gemm(gt, [(wt, out_f, out, out_f)], k, xq, n_tok, split=split)
        if split:  # second call on the same scratch
            out2 = cuda.empty_like(out)
            from qwen_haiku_b200 import GemmJob
            import ctypes as C
            arr = (GemmJob * 1)(GemmJob(wt.data_ptr(), out_f, out2.data_ptr(), out_f))
            cuda.cuda.synchronize()  # weights and activations complete: the early weight stream is allowed
            qh.check(qh.lib().qh_gemm(gt, C.cast(arr, C.c_void_p), 1, k, C.c_void_p(xq.data_ptr()), n_tok,
                                      C.c_void_p(scratch.data_ptr()), scratch.numel(), 1, None), "qh_gemm")
            cuda.cuda.synchronize()
            assert np.array_equal(bits(out2.cpu().numpy()), bits(out.cpu().numpy()))
            assert int(scratch[:4096].sum()) == 0, "split-K counters not reset"
        cuda.cuda.synchronize()
        outs.append(out.cpu().numpy())
    assert_bitwise(outs[1], outs[0], "split vs unsplit")
    assert_bitwise(outs[0], oracle.matmul(gt, w, out_f, k, x_np).reshape(n_tok, out_f), "oracle")


QH_GEMM_EXPANDED = 2


@pytest.mark.parametrize("gt", [Q4_K, Q5_K, Q6_K])
@pytest.mark.parametrize("k,out_f,n_tok", [(256, 128, 64), (1024, 300, 70), (2048, 257, 1), (3584, 1024, 64)])
@pytest.mark.parametrize("split", [False, True])
def test_expanded_weights_bitexact(qh, cuda, oracle, gt, k, out_f, n_tok, split):
    """qh_gemm on expanded weights (QH_GEMM_EXPANDED: the MMA operands
    streamed as stored, no expansion in the kernel) equals the oracle bit
    for bit, with and without split-K, and the tiled path."""
    w = qh.host.synth_blocks(gt, out_f * (k // 256), 0xE0 + gt + k + out_f)
    x_np = qh.host.synth_normal(n_tok * k, 0xE1 + k + n_tok).reshape(n_tok, k)
    wt = qh.host.gemm_pack(gt, qh.host.to_device(w), k, out_f)
    we = qh.host.gemm_expand(gt, wt, k, out_f)
    assert we.numel() == qh.lib().qh_gemm_expanded_bytes(gt, k, out_f)
    xq = qh.host.quantize_q8kt(qh.host.to_device(x_np), k, n_tok)
    a = cuda.empty((n_tok, out_f), dtype=cuda.float32, device="cuda")
    b = cuda.empty((n_tok, out_f), dtype=cuda.float32, device="cuda")
    qh.host.gemm(gt, [(wt, out_f, a, out_f)], k, xq, n_tok, split=split)
    qh.host.gemm(gt, [(we, out_f, b, out_f)], k, xq, n_tok, split=split, flags=QH_GEMM_EXPANDED)
    cuda.cuda.synchronize()
    want = oracle.matmul(gt, w, out_f, k, x_np).reshape(n_tok, out_f)
    assert_bitwise(b.cpu().numpy(), want, f"expanded type {gt} k={k} out_f={out_f} n={n_tok}")
    assert_bitwise(b.cpu().numpy(), a.cpu().numpy(), "expanded vs tiled")


@pytest.mark.parametrize("gt,k,out_f,n_tok", [(Q6_K, 3584, 1024, 64), (Q4_K, 2048, 1024, 64), (Q5_K, 2048, 257, 1)])
def test_expanded_split_spread_reduction(qh, cuda, oracle, gt, k, out_f, n_tok):
    """Expanded weights, few output tiles: every chunk's CTA of a tile waits
    for the others and sums a slice of the tile's elements in block order.
    Equal to the oracle bit for bit, on two calls over one scratch, and both
    arrival counters back at zero after each call."""
    w = qh.host.synth_blocks(gt, out_f * (k // 256), 0x5D + k + gt)
    x_np = qh.host.synth_normal(n_tok * k, 0x5E + k).reshape(n_tok, k)
    we = qh.host.gemm_expand(gt, qh.host.gemm_pack(gt, qh.host.to_device(w), k, out_f), k, out_f)
    xq = qh.host.quantize_q8kt(qh.host.to_device(x_np), k, n_tok)
    want = oracle.matmul(gt, w, out_f, k, x_np).reshape(n_tok, out_f)
    out = cuda.empty((n_tok, out_f), dtype=cuda.float32, device="cuda")
    scratch = qh.host.gemm(gt, [(we, out_f, out, out_f)], k, xq, n_tok, split=True, flags=QH_GEMM_EXPANDED)
    cuda.cuda.synchronize()
    assert_bitwise(out.cpu().numpy(), want, "first call")
    assert int(scratch[:4096].sum()) == 0, "split-K counters not reset"
    from qwen_haiku_b200 import GemmJob
    import ctypes as C
    out2 = cuda.full_like(out, -3.0)
    arr = (GemmJob * 1)(GemmJob(we.data_ptr(), out_f, out2.data_ptr(), out_f))
    qh.check(qh.lib().qh_gemm(gt, C.cast(arr, C.c_void_p), 1, k, C.c_void_p(xq.data_ptr()), n_tok,
                              C.c_void_p(scratch.data_ptr()), scratch.numel(), QH_GEMM_EXPANDED, None), "qh_gemm")
    cuda.cuda.synchronize()
    assert_bitwise(out2.cpu().numpy(), want, "second call on the same scratch")
    assert int(scratch[:4096].sum()) == 0, "split-K counters not reset"
    assert qh.lib().qh_check_device_error(None) == 0


def test_expanded_grouped_jobs(qh, cuda, oracle):
    """Three expanded Q4_K matrices in one launch, 130 tokens (3 token tiles)."""
    k, n_tok = 1024, 130
    x_np = qh.host.synth_normal(n_tok * k, 0xE7).reshape(n_tok, k)
    xq = qh.host.quantize_q8kt(qh.host.to_device(x_np), k, n_tok)
    jobs, ws, outs = [], [], []
    for i, out_f in enumerate((2048, 256, 16)):
        w = qh.host.synth_blocks(Q4_K, out_f * 4, 0xE8 + i)
        we = qh.host.gemm_expand(Q4_K, qh.host.gemm_pack(Q4_K, qh.host.to_device(w), k, out_f), k, out_f)
        out = cuda.empty((n_tok, out_f), dtype=cuda.float32, device="cuda")
        ws.append(w)
        outs.append((we, out))
        jobs.append((we, out_f, out, out_f))
    qh.host.gemm(Q4_K, jobs, k, xq, n_tok, flags=QH_GEMM_EXPANDED)
    cuda.cuda.synchronize()
    for (out_f, w, (_, out)) in zip((2048, 256, 16), ws, outs):
        assert_bitwise(out.cpu().numpy(), oracle.matmul(Q4_K, w, out_f, k, x_np).reshape(n_tok, out_f),
                       f"job {out_f}")


@pytest.mark.parametrize("cfg", ["3a", "3b"])
def test_prefill_configs(qh, cuda, oracle, cfg):
    """Benchmark config 3: M=512 K=1024 N=3584 Q4_K and M=2048 K=3584 N=1024
    Q6_K, full size on the GPU; the oracle checks a seeded subset of tokens
    (tokens are independent) bit for bit."""
    m, k, n, gt = (512, 1024, 3584, Q4_K) if cfg == "3a" else (2048, 3584, 1024, Q6_K)
    w = qh.host.synth_blocks(gt, n * (k // 256), 0x3A if cfg == "3a" else 0x3B)
    x = qh.host.synth_normal(m * k, 0x33 + m).reshape(m, k)
    got = run_gemm(qh, cuda, gt, w, k, n, x)
    rows = np.random.default_rng(3).choice(m, 24, replace=False)
    rows = np.unique(np.concatenate([rows, [0, 63, 64, m - 1]]))
    want = oracle.matmul(gt, w, n, k, x[rows]).reshape(len(rows), n)
    assert_bitwise(got[rows], want, f"config {cfg}")
    assert np.all(np.isfinite(got))


def test_gemm_rejects_q8_0_and_small_workspace(qh, cuda):
    L = qh.lib()
    assert L.qh_matmul_gemm_workspace_bytes(Q8_0, 1024, 64, 64) < 0
    import ctypes as C
    w = qh.host.to_device(qh.host.synth_blocks(Q4_K, 64 * 4, 1))
    x = qh.host.to_device(qh.host.synth_normal(64 * 1024, 2))
    out = cuda.empty((64, 64), dtype=cuda.float32, device="cuda")
    need = int(L.qh_matmul_gemm_workspace_bytes(Q4_K, 1024, 64, 64))
    work = cuda.empty(need, dtype=cuda.uint8, device="cuda")
    rc = L.qh_matmul_gemm(Q4_K, C.c_void_p(w.data_ptr()), 1024, 64, C.c_void_p(x.data_ptr()), 64,
                          C.c_void_p(out.data_ptr()), C.c_void_p(work.data_ptr()), need - 16, None)
    assert rc == -5  # QH_ERR_WORKSPACE
    rc = L.qh_matmul_gemm(Q8_0, C.c_void_p(w.data_ptr()), 1024, 64, C.c_void_p(x.data_ptr()), 64,
                          C.c_void_p(out.data_ptr()), C.c_void_p(work.data_ptr()), need, None)
    assert rc == -2  # QH_ERR_UNSUPPORTED


def test_quantize_q8kt_matches_split_layout(qh, cuda):
    """The tiled quantizer writes the same quants and scales as qh_quantize_q8k,
    and min-operand rows that encode the sub-block sums of the bsums."""
    k, n_tok = 1024, 70
    x_np = qh.host.synth_normal(n_tok * k, 9, 0.0, 3.0).reshape(n_tok, k)
    x = qh.host.to_device(x_np)
    split = qh.host.quantize_q8k(x, k, n_tok)
    tiled = qh.host.quantize_q8kt(x, k, n_tok)
    cuda.cuda.synchronize()
    qs, d, bs = qh.host.unpack_q8k(split.cpu().numpy(), k, n_tok)
    t = tiled.cpu().numpy()
    nb, tiles, TB = k // 256, (n_tok + 63) // 64, 18688
    assert t.size == tiles * nb * TB
    blk = t.reshape(tiles, nb, TB)
    q = blk[:, :, :16384].view(np.int8).reshape(tiles, nb, 16, 64, 16)
    q = q.transpose(0, 3, 1, 2, 4).reshape(tiles * 64, k)[:n_tok]
    assert np.array_equal(q, qs)
    dt = blk[:, :, 16384:16640].copy().view(np.float32).reshape(tiles, nb, 64).transpose(0, 2, 1)
    dt = dt.reshape(tiles * 64, nb)[:n_tok]
    assert np.array_equal(dt.view(np.uint32), np.asarray(d, np.float32).reshape(n_tok, nb).view(np.uint32))
    mn = blk[:, :, 16640:].view(np.int8).reshape(tiles, nb, 2, 64, 16).astype(np.int64)
    S = mn[:, :, 0, :, :8] + 128 * mn[:, :, 1, :, :8]               # [tiles, nb, 64, 8]
    S = S.transpose(0, 2, 1, 3).reshape(tiles * 64, nb, 8)[:n_tok]
    want = bs.reshape(n_tok, nb, 8, 2).astype(np.int64).sum(-1)
    assert np.array_equal(S, want)
    assert np.all(mn[:, :, :, :n_tok % 64 or 64, 8:] == 0)
