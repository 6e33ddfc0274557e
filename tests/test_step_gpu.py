# SPDX-License-Identifier: MIT
"""GPU: the persistent decode step (qh_step_create / qh_step_run,
include/qh_kernels.h; QH_DECODE_PERSISTENT, include/qh_slm.h) against the
launch-per-operation step it replaces. The bar is bit-identical outputs:
the phases run the same operations in the same order, only without a launch
between them."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q4_K, Q5_K, Q6_K = 12, 13, 14


def bits(t):
    import torch
    return t.view(torch.int32)


def make_program(qh, phases, d_pos):
    L = qh.lib()
    arr = (qh.StepPhase * len(phases))(*phases)
    prog = C.c_void_p()
    qh.check(L.qh_step_create(arr, len(phases), qh.host.dptr(d_pos), C.byref(prog)), "qh_step_create")
    return prog


def matvec_phase(qh, xform, k, xa, xb=None, xw=None, xh_out=None, eps=1e-6, projs=(), act=None):
    h = qh.host
    ph = qh.StepPhase()
    ph.kind = qh.STEP_MATVEC
    ph.xform = xform
    ph.xk = k
    ph.eps = eps
    ph.d_xa = xa.data_ptr()
    ph.d_xb = xb.data_ptr() if xb is not None else None
    ph.d_xw = xw.data_ptr() if xw is not None else None
    ph.d_xh_out = xh_out.data_ptr() if xh_out is not None else None
    ph.d_act_out = act.data_ptr() if act is not None else None
    ph.n_proj = len(projs)
    for i, (gt, w, out_f, out) in enumerate(projs):
        ph.proj[i].type = gt
        ph.proj[i].d_w = w.data_ptr()
        ph.proj[i].k = k
        ph.proj[i].out_f = out_f
        ph.proj[i].d_out = out.data_ptr()
    return ph


@pytest.mark.parametrize("paired", [False, True])
def test_matvec_phases_equal_separate_kernels(qh, cuda, paired):
    """Four dependent projection phases in ONE launch -- residual + RMSNorm
    into Q4_K gate/up (3584 rows each: several tiles per CTA), SwiGLU into a
    Q6_K down projection (1024 rows of 14 blocks: one split tile per CTA),
    residual + RMSNorm into a Q6_K head of 20000 rows (multi-group tiles, a
    ragged last tile), plain quantization into Q5_K (1024 and 40 rows) --
    equal, bit for bit, the separate kernels (qh_rmsnorm_q8k, qh_swiglu_q8k,
    qh_quantize_q8k, grouped matvec plans) run one after another; so do the
    residual sums the RMSNorm phases write. paired: the gate/up phase forms
    the SwiGLU row itself (d_act_out, equal to qh_swiglu's) and the down
    phase quantizes it."""
    torch = cuda
    h = qh.host
    L = qh.lib()
    H, F, V, K5 = 1024, 3584, 20000, 2048
    dev = lambda a: h.to_device(a)
    a = dev(h.synth_normal(H, 0x5101))
    b = dev(h.synth_normal(H, 0x5102, 0.0, 0.5))
    w1 = dev(h.synth_normal(H, 0x5103, 1.0, 0.02))
    w2 = dev(h.synth_normal(H, 0x5104, 1.0, 0.02))
    x5 = dev(h.synth_normal(K5, 0x5105))
    wg = dev(h.synth_blocks(Q4_K, F * H // 256, 0x5201))
    wu = dev(h.synth_blocks(Q4_K, F * H // 256, 0x5202))
    wd = dev(h.synth_blocks(Q6_K, H * F // 256, 0x5203))
    wh = dev(h.synth_blocks(Q6_K, V * H // 256, 0x5204))
    w5a = dev(h.synth_blocks(Q5_K, 1024 * K5 // 256, 0x5205))
    w5b = dev(h.synth_blocks(Q5_K, 40 * K5 // 256, 0x5206))
    f32 = lambda n: torch.full((n,), 3.0, dtype=torch.float32, device="cuda")
    pos = torch.zeros(4, dtype=torch.int32, device="cuda")

    # the separate kernels
    s = h.stream_handle()
    r = {n: f32(m) for n, m in (("g", F), ("u", F), ("d", H), ("h1", H), ("h2", H), ("v", V), ("p", 1024), ("q", 40))}
    xqH = torch.empty(int(L.qh_q8k_bytes(H, 1)), dtype=torch.uint8, device="cuda")
    xqF = torch.empty(int(L.qh_q8k_bytes(F, 1)), dtype=torch.uint8, device="cuda")
    xq5 = torch.empty(int(L.qh_q8k_bytes(K5, 1)), dtype=torch.uint8, device="cuda")
    qh.check(L.qh_rmsnorm_q8k(h.dptr(a), h.dptr(b), h.dptr(r["h1"]), h.dptr(w1), H, 1, 1e-6, h.dptr(xqH), 0, s), "rn")
    p1 = h.MatvecPlan(Q4_K, [(wg, xqH, r["g"], H, F), (wu, xqH, r["u"], H, F)], 1)
    p1.run()
    qh.check(L.qh_swiglu_q8k(h.dptr(r["g"]), h.dptr(r["u"]), F, 1, h.dptr(xqF), 0, s), "swiglu")
    p2 = h.MatvecPlan(Q6_K, [(wd, xqF, r["d"], F, H)], 1)
    p2.run()
    qh.check(L.qh_rmsnorm_q8k(h.dptr(r["h1"]), h.dptr(r["d"]), h.dptr(r["h2"]), h.dptr(w2), H, 1, 1e-6, h.dptr(xqH),
                              0, s), "rn2")
    p3 = h.MatvecPlan(Q6_K, [(wh, xqH, r["v"], H, V)], 1)
    p3.run()
    qh.check(L.qh_quantize_q8k(h.dptr(x5), K5, 1, h.dptr(xq5), s), "quantize")
    p4 = h.MatvecPlan(Q5_K, [(w5a, xq5, r["p"], K5, 1024), (w5b, xq5, r["q"], K5, 40)], 1)
    p4.run()
    torch.cuda.synchronize()

    # one program, one launch (and a second launch of the same program)
    g = {n: f32(m) for n, m in (("g", F), ("u", F), ("d", H), ("h1", H), ("h2", H), ("v", V), ("p", 1024), ("q", 40))}
    act_ref = f32(F)
    qh.check(L.qh_swiglu(h.dptr(r["g"]), h.dptr(r["u"]), h.dptr(act_ref), F, s), "swiglu")
    torch.cuda.synchronize()
    if paired:
        g["act"] = f32(F)
        r["act"] = act_ref
    phases = [
        matvec_phase(qh, qh.STEP_X_RESNORM, H, a, b, w1, g["h1"], projs=[(Q4_K, wg, F, g["g"]), (Q4_K, wu, F, g["u"])],
                     act=g.get("act")),
        matvec_phase(qh, qh.STEP_X_QUANT, F, g["act"], projs=[(Q6_K, wd, H, g["d"])]) if paired else
        matvec_phase(qh, qh.STEP_X_SWIGLU, F, g["g"], g["u"], projs=[(Q6_K, wd, H, g["d"])]),
        matvec_phase(qh, qh.STEP_X_RESNORM, H, g["h1"], g["d"], w2, g["h2"], projs=[(Q6_K, wh, V, g["v"])]),
        matvec_phase(qh, qh.STEP_X_QUANT, K5, x5, projs=[(Q5_K, w5a, 1024, g["p"]), (Q5_K, w5b, 40, g["q"])]),
    ]
    prog = make_program(qh, phases, pos)
    try:
        for run in range(2):
            for t in g.values():
                t.fill_(5.0)
            qh.check(L.qh_step_run(prog, 0, len(phases), s), "qh_step_run")
            torch.cuda.synchronize()
            qh.check(L.qh_check_device_error(None), "device error")
            for n in r:
                assert torch.equal(bits(g[n]), bits(r[n])), f"run {run}: {n} differs"
        # a program runs any range of its phases: the last two alone
        g["v"].fill_(5.0)
        g["p"].fill_(5.0)
        qh.check(L.qh_step_run(prog, 2, 2, s), "qh_step_run range")
        torch.cuda.synchronize()
        assert torch.equal(bits(g["v"]), bits(r["v"])) and torch.equal(bits(g["p"]), bits(r["p"]))
        assert L.qh_step_run(prog, 3, 2, s) != 0  # beyond the program
    finally:
        L.qh_step_destroy(prog)
        for p in (p1, p2, p3, p4):
            p.close()


def test_step_create_rejects_bad_phases(qh, cuda):
    torch = cuda
    h = qh.host
    L = qh.lib()
    x = h.to_device(h.synth_normal(1024, 1))
    out = torch.empty(64, dtype=torch.float32, device="cuda")
    w8 = h.to_device(h.synth_blocks(qh.Q8_0, 64 * 1024 // 32, 2))
    pos = torch.zeros(4, dtype=torch.int32, device="cuda")
    prog = C.c_void_p()
    bad_type = matvec_phase(qh, qh.STEP_X_QUANT, 1024, x, projs=[(qh.Q8_0, w8, 64, out)])
    arr = (qh.StepPhase * 1)(bad_type)
    assert L.qh_step_create(arr, 1, h.dptr(pos), C.byref(prog)) == -2  # QH_ERR_UNSUPPORTED
    w4 = h.to_device(h.synth_blocks(Q4_K, 64 * 4, 3))
    bad_k = matvec_phase(qh, qh.STEP_X_QUANT, 1000, x, projs=[(Q4_K, w4, 64, out)])
    arr = (qh.StepPhase * 1)(bad_k)
    assert L.qh_step_create(arr, 1, h.dptr(pos), C.byref(prog)) == -1  # QH_ERR_INVALID
    assert L.qh_step_create(arr, 0, h.dptr(pos), C.byref(prog)) == -1


def decode(slm, prompt, n_new):
    slm.reset()
    logits, picks = [], []
    tok = np.array([prompt[0]], np.int32)
    for pos in range(len(prompt) + n_new - 1):
        nxt, lg = slm.step(tok, pos, want_logits=True)
        picks.append(int(nxt[0]))
        logits.append(lg.copy())
        tok = np.array([prompt[pos + 1]], np.int32) if pos + 1 < len(prompt) else nxt
    return np.array(picks), np.stack(logits)


@pytest.mark.parametrize("full", [False, True])
def test_persistent_step_equals_launches(qh, cuda, full):
    """A whole model at one sequence (DeltaNet and attention layers, every
    projection, the head): QH_DECODE_PERSISTENT gives the logits of
    QH_DECODE_LAUNCHES bit for bit at every step (small model: 4 layers,
    32 steps; full BASELINE config-4 shape: 24 layers, 40 steps)."""
    h = qh.host
    cfg = h.slm_config(128) if full else h.slm_config(64, n_layers=4, vocab=4096)
    blob = h.Blob(cfg, 0xD15 + full)
    rng = np.random.default_rng(77 + full)
    prompt = rng.integers(0, cfg.vocab, 16 if full else 8).astype(np.int32)
    n_new = 24
    slm = h.Slm(cfg, blob, 1)
    slm.set_decode_mode(qh.DECODE_LAUNCHES)
    lp, ll = decode(slm, prompt, n_new)
    assert slm.decode_mode() == qh.DECODE_LAUNCHES
    slm.set_decode_mode(qh.DECODE_PERSISTENT)
    pp, pl = decode(slm, prompt, n_new)
    assert slm.decode_mode() == qh.DECODE_PERSISTENT, "the persistent step did not run"
    slm.close()
    assert np.array_equal(pp, lp)
    diff = [i for i in range(len(pl)) if not np.array_equal(pl[i].view(np.uint32), ll[i].view(np.uint32))]
    assert not diff, f"logits differ at steps {diff[:8]}"


def test_persistent_device_driven_and_sampled(qh, cuda):
    """begin/advance/picks (graph replays of the persistent step) and sampled
    generation give the same tokens in both decode modes."""
    h = qh.host
    cfg = h.slm_config(64, n_layers=4, vocab=4096)
    blob = h.Blob(cfg, 0xD17)
    rng = np.random.default_rng(78)
    prompt = rng.integers(0, cfg.vocab, (1, 9)).astype(np.int32)
    got = {}
    for mode in (qh.DECODE_LAUNCHES, qh.DECODE_PERSISTENT):
        slm = h.Slm(cfg, blob, 1)
        slm.set_decode_mode(mode)
        slm.begin(prompt)
        for n in (1, 5, 3, 12):
            slm.advance(n)
        picks = slm.picks(0, 21)
        sp = h.sampler_defaults()
        sampled = slm.generate_sampled(prompt, 16, sp, seeds=[1234])
        assert slm.decode_mode() == mode
        got[mode] = (picks, sampled[0])
        slm.close()
    assert np.array_equal(got[0][0], got[1][0]), "greedy picks differ between decode modes"
    assert np.array_equal(got[0][1], got[1][1]), "sampled tokens differ between decode modes"


def test_models_that_do_not_qualify_run_launches(qh, cuda):
    """Two sequences, or Q8_0 projections (the released Q4_K_M type mix), keep
    the launch-per-operation step."""
    h = qh.host
    cfg = h.slm_config(64, n_layers=4, vocab=4096)
    for n_seq, mix in ((2, 0), (1, 1)):
        blob = h.Blob(cfg, 0xD18, mix=mix)
        slm = h.Slm(cfg, blob, n_seq)
        slm.step(np.zeros(n_seq, np.int32), 0)
        assert slm.decode_mode() == qh.DECODE_LAUNCHES
        slm.close()


def test_step_timeout_is_reported_and_recovers(qh, cuda):
    """Failure detection without a fault: qh_step_test_timeout leaves out one
    tile's copy in CTA 0 with a short wait limit. The launch ends by itself
    (every wait is bounded; the other CTAs leave at their next grid barrier),
    qh_check_device_error reports QH_ERR_DEVICE once, and the same program
    then runs clean with the hook off, equal bit for bit to the separate
    kernels."""
    torch = cuda
    h = qh.host
    L = qh.lib()
    H, N1, N2 = 1024, 3000, 1024
    a = h.to_device(h.synth_normal(H, 0x7101))
    w = h.to_device(h.synth_normal(H, 0x7102, 1.0, 0.02))
    x2 = h.to_device(h.synth_normal(3584, 0x7103))
    w1 = h.to_device(h.synth_blocks(Q4_K, N1 * H // 256, 0x7201))
    w2 = h.to_device(h.synth_blocks(Q6_K, N2 * 3584 // 256, 0x7202))
    s = h.stream_handle()
    ref1 = torch.empty(N1, dtype=torch.float32, device="cuda")
    ref2 = torch.empty(N2, dtype=torch.float32, device="cuda")
    xq1 = torch.empty(int(L.qh_q8k_bytes(H, 1)), dtype=torch.uint8, device="cuda")
    xq2 = torch.empty(int(L.qh_q8k_bytes(3584, 1)), dtype=torch.uint8, device="cuda")
    qh.check(L.qh_rmsnorm_q8k(h.dptr(a), None, None, h.dptr(w), H, 1, 1e-6, h.dptr(xq1), 0, s), "rn")
    p1 = h.MatvecPlan(Q4_K, [(w1, xq1, ref1, H, N1)], 1)
    p1.run()
    qh.check(L.qh_quantize_q8k(h.dptr(x2), 3584, 1, h.dptr(xq2), s), "quantize")
    p2 = h.MatvecPlan(Q6_K, [(w2, xq2, ref2, 3584, N2)], 1)
    p2.run()
    torch.cuda.synchronize()
    out1 = torch.empty(N1, dtype=torch.float32, device="cuda")
    out2 = torch.empty(N2, dtype=torch.float32, device="cuda")
    pos = torch.zeros(4, dtype=torch.int32, device="cuda")
    phases = [matvec_phase(qh, qh.STEP_X_RESNORM, H, a, None, w, None, projs=[(Q4_K, w1, N1, out1)]),
              matvec_phase(qh, qh.STEP_X_QUANT, 3584, x2, projs=[(Q6_K, w2, N2, out2)])]
    prog = make_program(qh, phases, pos)
    try:
        assert L.qh_check_device_error(None) == 0
        qh.check(L.qh_step_test_timeout(prog, 1, 1 << 12), "qh_step_test_timeout")
        qh.check(L.qh_step_run(prog, 0, 2, s), "qh_step_run (tile withheld)")
        torch.cuda.synchronize()
        assert L.qh_check_device_error(None) == -6  # QH_ERR_DEVICE
        assert L.qh_check_device_error(None) == 0   # read and cleared
        qh.check(L.qh_step_test_timeout(prog, -1, 0), "qh_step_test_timeout off")
        for _ in range(2):
            out1.fill_(5.0)
            out2.fill_(5.0)
            qh.check(L.qh_step_run(prog, 0, 2, s), "qh_step_run")
            torch.cuda.synchronize()
            assert L.qh_check_device_error(None) == 0
            assert torch.equal(bits(out1), bits(ref1)) and torch.equal(bits(out2), bits(ref2))
    finally:
        L.qh_step_destroy(prog)
        p1.close()
        p2.close()
