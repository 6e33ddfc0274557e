# SPDX-License-Identifier: MIT
"""GPU parity of the quantized matmul path against the oracle and the
reference's golden outputs. Bar: bit-exact fp32 (the kernels reproduce the
reference's rounding order); integers and quantized bytes bit-exact."""
import glob
import hashlib
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14
BW = {Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_bitwise(got, want, what=""):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    if not np.array_equal(bits(got), bits(want)):
        bad = np.flatnonzero(bits(got).ravel() != bits(want).ravel())
        i = bad[0]
        rel = np.abs(got.ravel() - want.ravel()).max() / max(np.abs(want).max(), 1e-30)
        raise AssertionError(f"{what}: {bad.size} mismatches, first at {i}: got {got.ravel()[i]!r} "
                             f"want {want.ravel()[i]!r}; max rel {rel:.3e}")


def gpu_matmul(qh, cuda, gt, w_np, k, out_f, x_np):
    w = qh.host.to_device(w_np)
    x = qh.host.to_device(np.ascontiguousarray(x_np, np.float32))
    out = qh.host.matmul(gt, w, k, out_f, x, n_tok=x_np.shape[0])
    cuda.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_matmul_matches_reference_golden(path, qh, cuda):
    g = np.load(path)
    gt, k, out_f = int(g["gtype"]), int(g["k"]), int(g["out_f"])
    w = qh.host.synth_blocks(gt, out_f * (k // BW[gt]), int(g["wseed"]))
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(g["w_sha256"])
    out = gpu_matmul(qh, cuda, gt, w, k, out_f, g["x"])
    assert_bitwise(out, g["out"], os.path.basename(path))


@pytest.mark.parametrize("n_tok", [1, 2, 3, 8, 11])
@pytest.mark.parametrize("k", [256, 1024, 3584])
def test_quantize_q8k_bitexact(qh, cuda, oracle, k, n_tok):
    x = qh.host.synth_normal(n_tok * k, 1000 + k + n_tok, 0.0, 2.0).reshape(n_tok, k)
    x[0, :256] = 0.0
    x[-1, 3] = 9.0
    x[-1, 7] = -9.0  # magnitude tie: the first one sets the sign of the scale
    buf = qh.host.quantize_q8k(qh.host.to_device(x), k, n_tok)
    cuda.cuda.synchronize()
    qs, d, bs = qh.host.unpack_q8k(buf.cpu().numpy(), k, n_tok)
    oq, od, ob = oracle.quantize_q8k(x)
    assert np.array_equal(qs, oq)
    assert np.array_equal(bits(d), bits(od))
    assert np.array_equal(bs, ob)


@pytest.mark.parametrize("n_tok", [1, 4, 9])
@pytest.mark.parametrize("k", [32, 1024, 3584])
def test_quantize_q8_0_bitexact(qh, cuda, oracle, k, n_tok):
    x = qh.host.synth_normal(n_tok * k, 2000 + k + n_tok, 0.0, 2.0).reshape(n_tok, k)
    x[0, :32] = 0.0
    # exact halves: 127 * (j + 0.5) / 127-scale lands on .5 before roundf
    x[-1, :32] = np.arange(32, dtype=np.float32) - 15.5
    buf = qh.host.quantize_q8_0(qh.host.to_device(x), k, n_tok)
    cuda.cuda.synchronize()
    qs, d = qh.host.unpack_q8_0(buf.cpu().numpy(), k, n_tok)
    oq, od = oracle.quantize_q8_0(x)
    assert np.array_equal(qs, oq)
    assert np.array_equal(d, od)


SHAPES = [(256, 8), (256, 13), (1024, 3072), (1024, 1000), (2048, 256), (3584, 96), (1024, 9)]


@pytest.mark.parametrize("gt", [Q4_K, Q5_K, Q6_K, Q8_0])
@pytest.mark.parametrize("k,out_f", SHAPES)
@pytest.mark.parametrize("n_tok", [1, 2, 5, 8, 11])
def test_matmul_bitexact_vs_oracle(qh, cuda, oracle, gt, k, out_f, n_tok):
    w = qh.host.synth_blocks(gt, out_f * (k // BW[gt]), 31 * k + out_f + gt)
    x = qh.host.synth_normal(n_tok * k, 7 * k + n_tok).reshape(n_tok, k)
    out = gpu_matmul(qh, cuda, gt, w, k, out_f, x)
    assert_bitwise(out, oracle.matmul(gt, w, out_f, k, x), f"type {gt} k {k} out_f {out_f} n {n_tok}")


def test_per_type_entry_points(qh, cuda, oracle):
    k, out_f = 1024, 64
    x = qh.host.synth_normal(k, 5).reshape(1, k)
    xd = qh.host.to_device(x)
    for gt, fn in [(Q4_K, qh.host.tensor_matmul_q4k_f32), (Q5_K, qh.host.tensor_matmul_q5k_f32),
                   (Q6_K, qh.host.tensor_matmul_q6k_f32), (Q8_0, qh.host.tensor_matmul_q8_0_f32)]:
        w = qh.host.synth_blocks(gt, out_f * (k // BW[gt]), 50 + gt)
        out = fn(qh.host.to_device(w), out_f, k, xd)
        cuda.cuda.synchronize()
        assert_bitwise(out.cpu().numpy(), oracle.matmul(gt, w, out_f, k, x), f"type {gt}")


def test_layer_matvec_set_grouped(qh, cuda, oracle):
    """the Q4_K_M layer matvec set, one grouped launch per type."""
    torch = cuda
    hidden = 1024
    mats = [("q", Q4_K, 1024, 2048), ("k", Q4_K, 1024, 512), ("v", Q4_K, 1024, 512),
            ("gate", Q4_K, 1024, 3584), ("up", Q4_K, 1024, 3584),
            ("down", Q6_K, 3584, 1024), ("attn_out", Q5_K, 2048, 1024), ("sq8", Q8_0, 1024, 1024)]
    xs = {k: qh.host.synth_normal(k, 900 + k).reshape(1, k) for k in (1024, 2048, 3584)}
    by_type = {}
    for i, (name, gt, k, n) in enumerate(mats):
        w = qh.host.synth_blocks(gt, n * (k // BW[gt]), 0x600 + i)
        by_type.setdefault(gt, []).append((name, w, k, n))
    for gt, items in by_type.items():
        jobs, outs = [], []
        for name, w, k, n in items:
            xdev = qh.host.to_device(xs[k])
            xq = (qh.host.quantize_q8_0 if gt == Q8_0 else qh.host.quantize_q8k)(xdev, k, 1)
            out = torch.full((1, n), float("nan"), dtype=torch.float32, device="cuda")
            jobs.append((qh.host.to_device(w), xq, out, k, n))
            outs.append((name, w, k, n, out))
        plan = qh.host.MatvecPlan(gt, jobs, 1)
        plan.run()
        torch.cuda.synchronize()
        for name, w, k, n, out in outs:
            assert_bitwise(out.cpu().numpy(), oracle.matmul(gt, w, n, k, xs[k]), name)
        plan.close()
    assert qh.lib().qh_check_device_error(None) == 0


def test_grouped_plan_table_path(qh, cuda, oracle):
    """More jobs than fit in the kernel parameters -> device job table."""
    torch = cuda
    k, n_jobs = 1024, 20
    jobs, refs = [], []
    for i in range(n_jobs):
        n = 8 * (i + 1) + (i % 3)
        w = qh.host.synth_blocks(Q4_K, n * 4, 300 + i)
        x = qh.host.synth_normal(2 * k, 400 + i).reshape(2, k)
        xq = qh.host.quantize_q8k(qh.host.to_device(x), k, 2)
        out = torch.empty((2, n), dtype=torch.float32, device="cuda")
        jobs.append((qh.host.to_device(w), xq, out, k, n))
        refs.append((w, x, n, out))
    plan = qh.host.MatvecPlan(Q4_K, jobs, 2)
    plan.run()
    torch.cuda.synchronize()
    for w, x, n, out in refs:
        assert_bitwise(out.cpu().numpy(), oracle.matmul(Q4_K, w, n, k, x), f"n {n}")


def test_grouped_plan_rows_of_shared_buffer(qh, cuda, oracle):
    """Jobs reading different rows of ONE batched activation buffer."""
    torch = cuda
    k, G, n = 1024, 12, 136
    x = qh.host.synth_normal(G * k, 77).reshape(G, k)
    xq = qh.host.quantize_q8k(qh.host.to_device(x), k, G)
    jobs, refs = [], []
    for g in range(G):
        w = qh.host.synth_blocks(Q4_K, n * 4, 500 + g)
        out = torch.empty((1, n), dtype=torch.float32, device="cuda")
        jobs.append((qh.host.to_device(w), xq, out, k, n, G, g))
        refs.append((w, x[g:g + 1], out))
    plan = qh.host.MatvecPlan(Q4_K, jobs, 1)
    plan.run()
    torch.cuda.synchronize()
    for w, xg, out in refs:
        assert_bitwise(out.cpu().numpy(), oracle.matmul(Q4_K, w, n, k, xg), "shared buffer")


def test_lm_head_full_size_q6k(qh, cuda, oracle):
    """Largest matrix of the model: tied Q6_K head, 151936 x 1024."""
    k, out_f = 1024, 151936
    w = qh.host.synth_blocks(Q6_K, out_f * 4, 0xBEEF)
    x = qh.host.synth_normal(k, 0xFACE).reshape(1, k)
    out = gpu_matmul(qh, cuda, Q6_K, w, k, out_f, x)
    assert_bitwise(out, oracle.matmul(Q6_K, w, out_f, k, x), "lm head")


def test_misaligned_weight_rejected(qh, cuda):
    torch = cuda
    k, out_f = 256, 8
    w = torch.zeros(out_f * 144 + 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(k, dtype=torch.float32, device="cuda")
    out = torch.zeros(out_f, dtype=torch.float32, device="cuda")
    work = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    import ctypes as C
    rc = qh.lib().qh_matmul(Q4_K, C.c_void_p(w.data_ptr() + 2), k, out_f, C.c_void_p(x.data_ptr()), 1,
                            C.c_void_p(out.data_ptr()), C.c_void_p(work.data_ptr()), 4096, None)
    assert rc == -4


def test_no_device_error_reported(qh, cuda):
    assert qh.lib().qh_check_device_error(None) == 0


@pytest.mark.parametrize("gt,k", [(Q4_K, 1024), (Q5_K, 2048), (Q6_K, 3584), (Q4_K, 4096)])
@pytest.mark.parametrize("n_tok", [1, 3, 8])
def test_fused_input_equals_separate_kernels(qh, cuda, gt, k, n_tok):
    """qh_matvec_plan_fuse_input: the plan forming its own Q8_K input (residual
    + RMSNorm, SwiGLU, plain quantization) gives the same outputs, bit for bit,
    as the separate kernel followed by the plan; RMSNorm also writes h + b.
    Small and large launches (the split-tile path and the pipelined one)."""
    import ctypes as C
    torch = cuda
    h = qh.host
    L = qh.lib()
    outs = (40, 3000)  # 40 rows: one tile per CTA (split); 3000: several tiles per CTA
    a = h.to_device(h.synth_normal(n_tok * k, 0xF1 + k).reshape(n_tok, k))
    b = h.to_device(h.synth_normal(n_tok * k, 0xF2 + k, 0.0, 0.5).reshape(n_tok, k))
    w = h.to_device(h.synth_normal(k, 0xF3, 1.0, 0.02))
    ws = [h.to_device(h.synth_blocks(gt, n * (k // 256), 0xF4 + n)) for n in outs]
    xq = torch.empty(int(L.qh_q8k_bytes(k, n_tok)), dtype=torch.uint8, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for mode in (1, 2, 3, 4):  # 4: RMSNorm without a residual
        ref = [torch.empty((n_tok, n), dtype=torch.float32, device="cuda") for n in outs]
        got = [torch.empty((n_tok, n), dtype=torch.float32, device="cuda") for n in outs]
        h_ref = torch.empty_like(a)
        h_got = torch.full_like(a, 7.0)
        if mode == 1:
            qh.check(L.qh_rmsnorm_q8k(h.dptr(a), h.dptr(b), h.dptr(h_ref), h.dptr(w), k, n_tok, 1e-6, h.dptr(xq), 0, s),
                     "rmsnorm_q8k")
        elif mode == 2:
            qh.check(L.qh_swiglu_q8k(h.dptr(a), h.dptr(b), k, n_tok, h.dptr(xq), 0, s), "swiglu_q8k")
        elif mode == 3:
            qh.check(L.qh_quantize_q8k(h.dptr(a), k, n_tok, h.dptr(xq), s), "quantize_q8k")
        else:
            qh.check(L.qh_rmsnorm_q8k(h.dptr(a), None, None, h.dptr(w), k, n_tok, 1e-6, h.dptr(xq), 0, s),
                     "rmsnorm_q8k")
        plan_ref = h.MatvecPlan(gt, [(ws[i], xq, ref[i], k, n) for i, n in enumerate(outs)], n_tok)
        plan_ref.run()
        plan = h.MatvecPlan(gt, [(ws[i], xq, got[i], k, n) for i, n in enumerate(outs)], n_tok)
        if mode == 1:
            plan.fuse_input(1, a, b, w, 1e-6, h_got)
        elif mode == 2:
            plan.fuse_input(2, a, b)
        elif mode == 3:
            plan.fuse_input(3, a)
        else:
            plan.fuse_input(1, a, None, w, 1e-6, None)
        plan.run()
        torch.cuda.synchronize()
        for i in range(len(outs)):
            assert torch.equal(got[i].view(torch.int32), ref[i].view(torch.int32)), f"mode {mode} job {i}"
        if mode == 1:
            assert torch.equal(h_got.view(torch.int32), h_ref.view(torch.int32)), "residual h + b"
        plan.close()
        plan_ref.close()


@pytest.mark.parametrize("gt,no", [(Q4_K, 256), (Q4_K, 3072), (Q6_K, 1024)])
@pytest.mark.parametrize("n_tok", [1, 3])
def test_fused_output_tail_equals_separate_kernels(qh, cuda, gt, no, n_tok):
    """qh_matvec_plan_fuse_output: the launch's last CTA forms the next Q8_K
    rows from the plan's own outputs (residual + RMSNorm, SwiGLU of two jobs,
    plain quantization): the bytes equal the separate kernel's after the plan,
    the residual sum too; two launches in a row (the arrival counter is left
    at zero)."""
    import ctypes as C
    torch = cuda
    h = qh.host
    L = qh.lib()
    k = 1024
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    x = h.to_device(h.synth_normal(n_tok * k, 0xA1 + no).reshape(n_tok, k))
    xq_in = h.quantize_q8k(x, k, n_tok)
    ws = [h.to_device(h.synth_blocks(gt, no * (k // 256), 0xA2 + i)) for i in range(2)]
    hbase = h.to_device(h.synth_normal(n_tok * no, 0xA3 + no).reshape(n_tok, no))
    w = h.to_device(h.synth_normal(no, 0xA4, 1.0, 0.02))
    nbytes = int(L.qh_q8k_bytes(no, n_tok))
    for mode in (1, 2, 3):
        outs = [torch.empty((n_tok, no), dtype=torch.float32, device="cuda") for _ in range(2)]
        jobs = [(ws[i], xq_in, outs[i], k, no) for i in range(2 if mode == 2 else 1)]
        plan = h.MatvecPlan(gt, jobs, n_tok)
        xq_got = torch.full((nbytes,), 0x5A, dtype=torch.uint8, device="cuda")
        h_got = torch.full_like(hbase, 7.0)
        if mode == 1:
            plan.fuse_output(1, no, xq_got, hbase, outs[0], w, 1e-6, h_got)
        elif mode == 2:
            plan.fuse_output(2, no, xq_got, outs[0], outs[1])
        else:
            plan.fuse_output(3, no, xq_got, outs[0])
        for rep in range(2):
            xq_got.fill_(0x5A)
            plan.run()
            torch.cuda.synchronize()
            xq_ref = torch.full((nbytes,), 0x5A, dtype=torch.uint8, device="cuda")
            h_ref = torch.empty_like(hbase)
            if mode == 1:
                qh.check(L.qh_rmsnorm_q8k(h.dptr(hbase), h.dptr(outs[0]), h.dptr(h_ref), h.dptr(w), no, n_tok, 1e-6,
                                          h.dptr(xq_ref), 0, s), "rmsnorm_q8k")
            elif mode == 2:
                qh.check(L.qh_swiglu_q8k(h.dptr(outs[0]), h.dptr(outs[1]), no, n_tok, h.dptr(xq_ref), 0, s),
                         "swiglu_q8k")
            else:
                qh.check(L.qh_quantize_q8k(h.dptr(outs[0]), no, n_tok, h.dptr(xq_ref), s), "quantize_q8k")
            torch.cuda.synchronize()
            # compare the planes the quantizers define (the scale rows' padding aside)
            qs_ref, d_ref, bs_ref = h.unpack_q8k(xq_ref.cpu().numpy(), no, n_tok)
            qs_got, d_got, bs_got = h.unpack_q8k(xq_got.cpu().numpy(), no, n_tok)
            assert np.array_equal(qs_got, qs_ref), f"mode {mode} launch {rep}: quants"
            assert np.array_equal(d_got.view(np.uint32), d_ref.view(np.uint32)), f"mode {mode} launch {rep}: scales"
            assert np.array_equal(bs_got, bs_ref), f"mode {mode} launch {rep}: block sums"
            if mode == 1:
                assert torch.equal(h_got.view(torch.int32), h_ref.view(torch.int32)), "residual h + b"
        assert L.qh_check_device_error(None) == 0
        plan.close()


@pytest.mark.parametrize("k,out_f,n_tok", [(64, 16, 1), (1024, 300, 3), (100, 33, 11)])
def test_f32_weights_match_reference(qh, cuda, oracle, ref, k, out_f, n_tok):
    """matmul_dispatch's F32 case (tensor_matmul_f32, slm/tensor.c:517):
    float product and float add per element in index order."""
    rng = np.random.default_rng(k + out_f)
    w = rng.standard_normal((out_f, k)).astype(np.float32)
    x = rng.standard_normal((n_tok, k)).astype(np.float32)
    out = gpu_matmul(qh, cuda, 0, w.view(np.uint8).ravel(), k, out_f, x)
    assert_bitwise(out, ref.matmul(0, w.view(np.uint8).ravel(), out_f, k, x), "f32 vs reference")
    assert_bitwise(out, oracle.matmul(0, w.view(np.uint8).ravel(), out_f, k, x), "f32 vs oracle")


@pytest.mark.parametrize("n_tok", [9, 17, 64, 70])
def test_q8_0_many_tokens_bitexact(qh, cuda, oracle, n_tok):
    """Q8_0 weights for more than 8 tokens (one launch over every token)."""
    k, out_f = 1024, 48
    w = qh.host.synth_blocks(Q8_0, out_f * (k // 32), 0x80 + n_tok)
    x = qh.host.synth_normal(n_tok * k, 0x81 + n_tok).reshape(n_tok, k)
    assert_bitwise(gpu_matmul(qh, cuda, Q8_0, w, k, out_f, x), oracle.matmul(Q8_0, w, out_f, k, x), "q8_0 many")
