# SPDX-License-Identifier: MIT
"""Measures the constants that make the device expf/logf of
qwen.haiku_b200/csrc/qh_libm.cuh bit-identical to the host C library's
expf/logf, and writes them to qwen.haiku_b200/csrc/qh_libm_consts.h.

BUILD-TIME / TEST INFRASTRUCTURE (run by hand on an x86-64 Linux host with
the same C library the reference is built against; the GPU box never runs
it). Method, per function (libm_fit.c describes the evaluation structure):

1. Start from textbook values: Taylor coefficients of 2^(r/32) for expf;
   for logf the subinterval centres c_i (c = 1 for the subinterval holding
   1.0), log(c_i) in extended precision, and a least-squares quadratic q.
2. Cutting planes: evaluate the candidate on every float input, collect the
   inputs where it differs from the host library, turn each into linear
   bounds on the parameter change (the host's result fixes an interval of
   doubles the candidate must round from), and solve a linear program that
   maximises the smallest slack; re-linearise at the new point and repeat.
   Changes that add mismatches are rejected and the trust region shrinks.
   For logf: the polynomial first (from the subinterval with c = 1, where
   the table pair is exactly (1, 0)), then each table pair, then all
   parameters together, then single-ulp moves of what still mismatches.
3. Check all 2^32 inputs; write the header only if nothing differs.

    python oracle/libm/fit.py [--state _work/libm_fit.json]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import struct
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(ROOT, "qwen.haiku_b200", "csrc", "qh_libm_consts.h")
LD = np.longdouble


def _lib(build_dir):
    so = os.path.join(build_dir, "liblibmfit.so")
    src = os.path.join(HERE, "libm_fit.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        os.makedirs(build_dir, exist_ok=True)
        subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-o", so, src, "-lm"],
                       check=True)
    L = C.CDLL(so)
    i64, p = C.c_int64, C.c_void_p
    L.exp_rows.restype = i64
    L.exp_rows.argtypes = [p, p, p, p, p, i64, C.POINTER(i64)]
    L.log_rows.restype = i64
    L.log_rows.argtypes = [p, C.c_uint, p, p, p, p, i64, C.POINTER(i64)]
    L.log_rows_near.restype = i64
    L.log_rows_near.argtypes = [p, C.c_uint, C.c_double, p, p, p, p, i64, C.POINTER(i64)]
    L.exp_count_all.restype = i64
    L.exp_count_all.argtypes = [p, p]
    L.log_count_all.restype = i64
    L.log_count_all.argtypes = [p]
    L.set_log_exceptions.restype = None
    L.set_log_exceptions.argtypes = [p, p, C.c_int]
    return L


def _lp(A, b, nvar, bounds):
    from scipy.optimize import linprog
    cobj = np.zeros(nvar + 1)
    cobj[-1] = -1
    res = linprog(cobj, A_ub=A, b_ub=b, bounds=bounds, method="highs")
    return res.x if res.status == 0 else None


def exp2_table():
    """bits(2^(i/32)) rounded to nearest, minus i << 47 (the exponent the
    evaluation adds back), from the definition in 200-bit arithmetic."""
    import mpmath
    mpmath.mp.prec = 200
    out = []
    for i in range(32):
        d = float(mpmath.mpf(2) ** (mpmath.mpf(i) / 32))
        out.append(struct.unpack("<Q", struct.pack("<d", d))[0] - (i << 47))
    return np.array(out, np.uint64)


def fit_expf(L, log=print):
    tab = exp2_table()
    ln2 = np.log(2.0)
    orig = np.array([ln2 ** 3 / 6 / 32 ** 3, ln2 ** 2 / 2 / 32 ** 2, ln2 / 32])
    p = orig.copy()
    Rs, Ls, Us = [], [], []
    maxn = 2_000_000
    for it in range(40):
        R, Lb, Ub = np.zeros(maxn), np.zeros(maxn), np.zeros(maxn)
        n = C.c_int64()
        mis = L.exp_rows(p.ctypes.data, tab.ctypes.data, R.ctypes.data, Lb.ctypes.data, Ub.ctypes.data, maxn,
                         C.byref(n))
        log(f"expf it {it}: {mis} mismatches")
        if mis == 0:
            break
        k = min(n.value, maxn)
        R, Lb, Ub = R[:k], Lb[:k], Ub[:k]
        d = (p - orig) * 2.0 ** 60  # bounds relative to the fixed origin
        sh = d[2] * R + d[1] * R ** 2 + d[0] * R ** 3
        Lb, Ub = Lb + sh, Ub + sh
        if k > 200000:
            idx = np.random.default_rng(it).choice(k, 200000, replace=False)
            R, Lb, Ub = R[idx], Lb[idx], Ub[idx]
        Rs.append(R); Ls.append(Lb); Us.append(Ub)
        RR, LL, UU = np.concatenate(Rs), np.concatenate(Ls), np.concatenate(Us)
        phi = np.stack([RR ** 3, RR ** 2, RR], 1)
        a = np.abs(RR)[:, None]
        A = np.vstack([np.hstack([-phi, a]), np.hstack([phi, a])])
        x = _lp(A, np.concatenate([-LL, UU]), 3, [(None, None)] * 3 + [(None, 1e6)])
        if x is None:
            raise RuntimeError("expf: linear program infeasible")
        p = orig + x[:3] / 2.0 ** 60
    total = L.exp_count_all(p.ctypes.data, tab.ctypes.data)
    log(f"expf: {total} of 2^32 inputs differ from the host library")
    return p, tab, total


# ---- logf -------------------------------------------------------------------
OFF = 0x3f330000


def _f32(b):
    return struct.unpack("<f", struct.pack("<I", b))[0]


def log_init():
    th = np.zeros(36)
    for i in range(16):
        lo, hi = _f32(OFF + i * 2 ** 19), _f32(OFF + (i + 1) * 2 ** 19 - 1)
        c = 1.0 if i == 9 else (lo + hi) / 2
        th[i] = 1.0 / c
        th[16 + i] = float(np.log(LD(c)))
    r = np.linspace(-0.0315, 0.0315, 20001)
    r = r[r != 0]
    y = (np.log1p(r.astype(LD)) - r).astype(np.float64)
    M = np.stack([r ** 4, r ** 3, r ** 2], 1)
    w = 1 / np.abs(r)
    th[32:35] = np.linalg.lstsq(M * w[:, None], y * w, rcond=None)[0]
    th[35] = np.log(2.0)
    return th


def log_collect(L, th, mask, maxn=2_000_000, margin=0.0):
    I, K = np.zeros(maxn, np.int32), np.zeros(maxn, np.int32)
    Z, G = np.zeros(maxn), np.zeros(maxn, np.float32)
    n = C.c_int64()
    mis = L.log_rows_near(th.ctypes.data, mask, margin, I.ctypes.data, K.ctypes.data, Z.ctypes.data,
                          G.ctypes.data, maxn, C.byref(n))
    k = min(n.value, maxn)
    return mis, (I[:k], K[:k], Z[:k], G[:k])


def log_step(th, rows, var, scale):
    """One linear program over the rows at the current point; None if infeasible."""
    I, K, Z, G = rows
    gm, gp = np.nextafter(G, np.float32(-np.inf)), np.nextafter(G, np.float32(np.inf))
    lo, hi = (LD(1) * G + gm) / 2, (LD(1) * G + gp) / 2
    rr = LD(1) * Z * th[I] - 1
    y = LD(1) * th[16 + I] + K * LD(th[35]) + rr + rr * rr * (LD(th[34]) + LD(th[33]) * rr + LD(th[32]) * rr * rr)
    Lb = np.asarray((lo - y) * LD(2.0 ** 60), np.float64)
    Ub = np.asarray((hi - y) * LD(2.0 ** 60), np.float64)
    r = rr.astype(np.float64)
    m = len(I)
    J = np.zeros((m, 36))
    A0, A1, A2 = th[32], th[33], th[34]
    J[np.arange(m), I] = Z * (1 + 2 * A2 * r + 3 * A1 * r ** 2 + 4 * A0 * r ** 3)
    J[np.arange(m), 16 + I] = 1.0
    J[:, 32], J[:, 33], J[:, 34] = r ** 4, r ** 3, r ** 2
    J = J[:, var] * scale[var]  # variables: change / scale, in [-1, 1]
    w = np.abs(np.asarray((hi - lo) * LD(2.0 ** 60), np.float64))[:, None]
    A = np.vstack([np.hstack([-J, w]), np.hstack([J, w])])
    x = _lp(A, np.concatenate([-Lb, Ub]), len(var), [(-1, 1)] * len(var) + [(None, 0.5)])
    if x is None:
        return None
    th2 = th.copy()
    th2[var] += x[:len(var)] * scale[var] / 2.0 ** 60
    return th2


def log_fit(L, th, mask, var, scale, iters, label, log, new_cap=4000, acc_cap=40000):
    acc = None
    mis, rows = log_collect(L, th, mask)
    for it in range(iters):
        log(f"logf {label} it {it}: {mis} mismatches")
        if mis == 0:
            break
        rng = np.random.default_rng(it)
        if len(rows[0]) > new_cap:
            idx = rng.choice(len(rows[0]), new_cap, replace=False)
            rows = tuple(a[idx] for a in rows)
        acc = rows if acc is None else tuple(np.concatenate([a, b]) for a, b in zip(acc, rows))
        if len(acc[0]) > acc_cap:
            idx = rng.choice(len(acc[0]), acc_cap, replace=False)
            acc = tuple(a[idx] for a in acc)
        th2 = log_step(th, acc, var, scale)
        if th2 is None:
            scale = scale * 0.5
            continue
        mis2, rows2 = log_collect(L, th2, mask)
        if mis2 > mis:
            scale = scale * 0.5
            acc = tuple(np.concatenate([a, b[:new_cap]]) for a, b in zip(acc, rows2))
            continue
        th, mis, rows = th2, mis2, rows2
    return th, mis


def log_scan_c(L, th, i, log):
    """c_i (with log c_i in extended precision) of fewest mismatches on a
    grid around the current value, refined three times."""
    c0, span = 1 / th[i], 0.03
    for _ in range(4):
        best = None
        for d in np.linspace(-span, span, 41):
            c = c0 * (1 + d)
            t = th.copy()
            t[i], t[16 + i] = 1 / c, float(np.log(LD(c)))
            mis, _ = log_collect(L, t, 1 << i, maxn=1)
            if best is None or mis < best[0]:
                best = (mis, c)
        c0, span = best[1], span / 20
        log(f"logf i={i} scan: c {c0:.9f}, {best[0]} mismatches")
    th = th.copy()
    th[i], th[16 + i] = 1 / c0, float(np.log(LD(c0)))
    return th


def log_joint_near(L, th, log, margin=2e-6, iters=30):
    """All parameters at once against the mismatching inputs AND the matching
    ones within `margin` ulps of a rounding boundary, so that a step cannot
    break what it does not see; the trust region shrinks on rejection."""
    var = np.array([i for i in range(16) if i != 9] + [16 + i for i in range(16) if i != 9] + [32, 33, 34])
    scale = np.zeros(36)
    scale[:16], scale[16:32] = 1e-12 * th[:16], 1e-12
    scale[32], scale[33], scale[34] = 1e-8, 1e-9, 1e-10
    scale *= 2.0 ** 60
    mis, rows = log_collect(L, th, 0xffff, margin=margin)
    for it in range(iters):
        log(f"logf joint+near it {it}: {mis} mismatches, {len(rows[0])} rows")
        if mis == 0:
            break
        th2 = log_step(th, rows, var, scale)
        if th2 is None:
            scale = scale * 0.5
            continue
        mis2, rows2 = log_collect(L, th2, 0xffff, margin=margin)
        if mis2 >= mis:
            scale = scale * 0.5
            continue
        th, mis, rows = th2, mis2, rows2
    return th


def _ulp_move(x, n):
    return float(np.nextafter(x, np.inf if n > 0 else -np.inf)) if n else x


def log_polish(L, th, log):
    """Single-ulp moves while they remove mismatches: each table pair checked
    on its own subinterval, then the polynomial on all of them."""
    total, rows = log_collect(L, th, 0xffff)
    for rnd in range(20):
        if total == 0:
            break
        before = total
        for i in sorted(set(int(v) for v in rows[0])):
            mis, _ = log_collect(L, th, 1 << i, maxn=1)
            for j in (16 + i, i):
                for step in (1, -1):
                    while mis:
                        t2 = th.copy()
                        t2[j] = _ulp_move(t2[j], step)
                        m2, _ = log_collect(L, t2, 1 << i, maxn=1)
                        if m2 >= mis:
                            break
                        th, mis = t2, m2
        total, rows = log_collect(L, th, 0xffff)
        for j in (32, 33, 34):
            for step in (1, -1):
                while total:
                    t2 = th.copy()
                    t2[j] = _ulp_move(t2[j], step)
                    m2, r2 = log_collect(L, t2, 0xffff)
                    if m2 >= total:
                        break
                    th, total, rows = t2, m2, r2
        log(f"logf polish round {rnd}: {total} mismatches")
        if total >= before:
            break
    return th, total


def fit_logf(L, th=None, stage=0, save=None, log=print):
    if th is None:
        th = log_init()
    if stage <= 0:
        scale = np.ones(36) * 2.0 ** 60
        scale[32], scale[33], scale[34] = 1e-2 * 2 ** 60, 1e-3 * 2 ** 60, 1e-4 * 2 ** 60
        th, _ = log_fit(L, th, 1 << 9, np.array([32, 33, 34]), scale, 40, "poly (i=9)", log)
        save and save(th, 1)
    if stage <= 1:
        for i in [j for j in range(16) if j != 9]:
            scale = np.ones(36) * 2.0 ** 60
            scale[i], scale[16 + i] = 1e-4 * th[i] * 2 ** 60, 1e-4 * 2 ** 60
            th, m = log_fit(L, th, 1 << i, np.array([i, 16 + i]), scale, 25, f"i={i}", log)
            if m > 100:  # the table's c_i is further from the centre: scan for it, then fit again
                th = log_scan_c(L, th, i, log)
                th, m = log_fit(L, th, 1 << i, np.array([i, 16 + i]), scale, 25, f"i={i}", log)
            save and save(th, 1)
        save and save(th, 2)
    if stage <= 2:
        var = np.array([i for i in range(16) if i != 9] + [16 + i for i in range(16) if i != 9] + [32, 33, 34])
        scale = np.zeros(36)
        scale[:16], scale[16:32] = 1e-8 * th[:16], 1e-8
        scale[32], scale[33], scale[34] = 1e-6, 1e-7, 1e-8
        th, m = log_fit(L, th, 0xffff, var, scale * 2.0 ** 60, 150, "joint", log, 3000, 60000)
        save and save(th, 3)
    if stage <= 3:
        th = log_joint_near(L, th, log)
        save and save(th, 4)
    th, m = log_polish(L, th, log)
    save and save(th, 5)
    # What the fit leaves (inputs whose unrounded value lies within ~1e-6 ulp
    # of a rounding boundary, where no parameter set near this one rounds
    # every such input as the host does) is listed with the host's results.
    exc = _log_exception_list(L, th)
    log(f"logf: {len(exc)} inputs listed with the host's results")
    ein = np.array([e[0] for e in exc], np.uint32)
    eout = np.array([e[1] for e in exc], np.uint32)
    L.set_log_exceptions(ein.ctypes.data, eout.ctypes.data, len(exc))
    total = L.log_count_all(th.ctypes.data)
    log(f"logf: {total} of 2^32 inputs differ from the host library")
    save and save(th, 5, log_exceptions=[[hex(a), hex(b)] for a, b in exc])
    return th, total


def _log_exception_list(L, th):
    """(input bits, host result bits) of every positive finite input where the
    candidate differs from the host library, sorted by input."""
    import ctypes.util
    libm = C.CDLL(ctypes.util.find_library("m"))
    libm.logf.restype, libm.logf.argtypes = C.c_float, [C.c_float]
    I, K, Z, G = log_collect(L, th, 0xffff)[1]
    out = []
    for z, k, g in zip(Z, K, G):
        # the input is z * 2^k (z in [0x3f330000, 0x3f330000 + 2^23) as bits)
        zb = int(np.float32(z).view(np.uint32))
        if -126 <= int(k) + ((zb >> 23) - 127) <= 127:
            xb = zb + (int(k) << 23)
        else:  # subnormal input: z * 2^k is exact in float
            xb = int(np.float32(np.float64(z) * 2.0 ** int(k)).view(np.uint32))
        x = np.uint32(xb).view(np.float32)
        assert np.float32(libm.logf(float(x))).view(np.uint32) == np.float32(g).view(np.uint32)
        out.append((xb, int(np.float32(g).view(np.uint32))))
    return sorted(out)


def _hex(x):
    return float(x).hex()


def write_header(p, tab, th, exc):
    lines = [
        "// SPDX-License-Identifier: MIT",
        "//",
        "// qh_libm_consts.h -- GENERATED by oracle/libm/fit.py; do not edit.",
        "// Constants of the device expf/logf (qh_libm.cuh), measured against the",
        f"// host C library ({_libc()}): with them the device functions equal",
        "// the host's expf/logf on all 2^32 float inputs.",
        "",
        "#ifndef QH_LIBM_CONSTS_H",
        "#define QH_LIBM_CONSTS_H",
        "",
        "#include <stdint.h>",
        "",
        "namespace qh {",
        "namespace libm {",
        "",
        "// expf: 2^(i/32) rounded to nearest, as bits, minus i << 47.",
        "static __device__ const uint64_t kExp2Tab[32] = {",
    ]
    for i in range(0, 32, 4):
        lines.append("    " + ", ".join(f"0x{int(v):016x}ull" for v in tab[i:i + 4]) + ",")
    lines += [
        "};",
        "// expf: p(r) = 1 + kExpC2 r + kExpC1 r^2 + kExpC0 r^3, r = x 32/ln2 - k.",
        f"constexpr double kExpC0 = {_hex(p[0])}, kExpC1 = {_hex(p[1])}, kExpC2 = {_hex(p[2])};",
        "",
        "// logf: per subinterval i of the reduced argument, 1/c_i and log c_i.",
        "static __device__ const double kLogInvC[16] = {",
    ]
    for i in range(0, 16, 4):
        lines.append("    " + ", ".join(_hex(v) for v in th[i:i + 4]) + ",")
    lines += ["};", "static __device__ const double kLogLogC[16] = {"]
    for i in range(16, 32, 4):
        lines.append("    " + ", ".join(_hex(v) for v in th[i:i + 4]) + ",")
    lines += [
        "};",
        "// logf: log(1 + r) ~ r + r^2 (kLogA2 + kLogA1 r + kLogA0 r^2).",
        f"constexpr double kLogA0 = {_hex(th[32])}, kLogA1 = {_hex(th[33])}, kLogA2 = {_hex(th[34])};",
        f"constexpr double kLn2 = {_hex(th[35])};",
        "// logf: inputs (bits, ascending) whose result the fitted evaluation rounds",
        "// the other way than the host library, and the host's results.",
        f"constexpr int kLogExcN = {len(exc)};",
        "static __device__ const uint32_t kLogExcIn[kLogExcN > 0 ? kLogExcN : 1] = {"
        + ", ".join(f"0x{a:08x}u" for a, _ in exc) + "};",
        "static __device__ const uint32_t kLogExcOut[kLogExcN > 0 ? kLogExcN : 1] = {"
        + ", ".join(f"0x{b:08x}u" for _, b in exc) + "};",
        "",
        "}  // namespace libm",
        "}  // namespace qh",
        "",
        "#endif  // QH_LIBM_CONSTS_H",
        "",
    ]
    with open(OUT, "w") as f:
        f.write("\n".join(lines))


def _libc():
    import platform
    name, ver = platform.libc_ver()
    return f"{name} {ver}, x86-64 FMA variant"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--state", default=os.path.join(ROOT, "_work", "libm_fit.json"))
    ap.add_argument("--build-dir", default=os.path.join(ROOT, "_build", "libm"))
    ap.add_argument("--write-only", action="store_true", help="write the header from a finished state file")
    args = ap.parse_args()
    st = json.load(open(args.state)) if os.path.exists(args.state) else {}
    if args.write_only:
        write_header(np.array([float.fromhex(v) for v in st["expf"]]), exp2_table(),
                     np.array([float.fromhex(v) for v in st["th"]]),
                     [(int(a, 16), int(b, 16)) for a, b in st.get("log_exceptions", [])])
        print("wrote", OUT)
        return
    L = _lib(args.build_dir)

    def save(th=None, stage=None, **kw):
        if th is not None:
            st["th"], st["log_stage"] = [float(v).hex() for v in th], stage
        st.update(kw)
        os.makedirs(os.path.dirname(args.state), exist_ok=True)
        json.dump(st, open(args.state, "w"))

    def log(msg):
        print(msg, flush=True)

    if "expf" not in st:
        p, tab, total = fit_expf(L, log)
        if total:
            sys.exit("expf: no exact fit")
        save(expf=[float(v).hex() for v in p])
    p = np.array([float.fromhex(v) for v in st["expf"]])
    tab = exp2_table()
    th = np.array([float.fromhex(v) for v in st["th"]]) if "th" in st else None
    th, total = fit_logf(L, th, st.get("log_stage", 0), save, log)
    if total:
        sys.exit(f"logf: {total} inputs still differ; header not written")
    write_header(p, tab, th, [(int(a, 16), int(b, 16)) for a, b in st.get("log_exceptions", [])])
    print("wrote", OUT)


if __name__ == "__main__":
    main()
