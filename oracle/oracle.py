# SPDX-License-Identifier: MIT
"""ctypes loaders for the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
``--impl reference`` legs use this module, and only as the checker or the
timed CPU baseline; the qwen.haiku_b200 package never imports it.

  Oracle -- oracle/liboracle.so, this repository's C restatement
            (oracle/qh_oracle.c) of the reference's quantizers and dots.
  Ref    -- oracle/_ref/libqhref.so, the reference's own C sources compiled
            where they lie (oracle/ref_harness.c + oracle/Makefile).

Activation rows are passed as split planes (qs int8 [n, k], d f32 [n, k/256],
bsums int16 [n, k/256, 16]); ``to_q8k_blocks`` packs them into the
reference's 292-byte q8k_block array (simd/quants.h:94-99).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libqhref.so")

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_0: 34}
BLOCK_WEIGHTS = {Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_0: 32}

_P, _I, _I64, _F = C.c_void_p, C.c_int, C.c_int64, C.c_float


def reference_root():
    """The reference's source tree: $QH_REF_ROOT, else a directory named
    `reference` beside this repository; None when neither exists (test
    machines use the prebuilt _ref/ libraries)."""
    for cand in (os.environ.get("QH_REF_ROOT"), os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "slm")):
            return cand
    return None


def build(force: bool = False) -> None:
    """make -C oracle (liboracle.so; _ref/libqhref.so when the reference exists)."""
    if force or not os.path.exists(ORACLE_SO):
        root = reference_root()
        subprocess.run(["make", "-s", "-C", HERE] + ([f"REF_ROOT={root}"] if root else []), check=True)


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def to_q8k_blocks(qs: np.ndarray, d: np.ndarray, bs: np.ndarray) -> np.ndarray:
    """Split planes of ONE row -> q8k_block[k/256] bytes (292 B each)."""
    nb = d.shape[-1]
    out = np.zeros((nb, 292), dtype=np.uint8)
    out[:, 0:4] = np.ascontiguousarray(d.reshape(nb).astype(np.float32)).view(np.uint8).reshape(nb, 4)
    out[:, 4:260] = qs.reshape(nb, 256).view(np.uint8)
    out[:, 260:292] = np.ascontiguousarray(bs.reshape(nb, 16).astype(np.int16)).view(np.uint8).reshape(nb, 32)
    return out.reshape(-1)


def from_q8k_blocks(raw: np.ndarray, k: int):
    nb = k // 256
    r = raw.reshape(nb, 292)
    d = np.ascontiguousarray(r[:, 0:4]).view(np.float32).reshape(nb)
    qs = np.ascontiguousarray(r[:, 4:260]).view(np.int8).reshape(k)
    bs = np.ascontiguousarray(r[:, 260:292]).view(np.int16).reshape(nb, 16)
    return qs, d, bs


def to_q8_0_blocks(qs: np.ndarray, dbits: np.ndarray) -> np.ndarray:
    nb = dbits.shape[-1]
    out = np.zeros((nb, 34), dtype=np.uint8)
    out[:, 0:2] = np.ascontiguousarray(dbits.reshape(nb).astype(np.uint16)).view(np.uint8).reshape(nb, 2)
    out[:, 2:34] = qs.reshape(nb, 32).view(np.uint8)
    return out.reshape(-1)


def from_q8_0_blocks(raw: np.ndarray, k: int):
    nb = k // 32
    r = raw.reshape(nb, 34)
    return (np.ascontiguousarray(r[:, 2:34]).view(np.int8).reshape(k),
            np.ascontiguousarray(r[:, 0:2]).view(np.uint16).reshape(nb))


class Oracle:
    """This repository's CPU restatement (oracle/qh_oracle.c)."""

    def __init__(self):
        build()
        L = C.CDLL(ORACLE_SO)
        L.orc_quantize_row_q8k.argtypes = [_P, _I64, _P, _P, _P]
        L.orc_quantize_row_q8_0.argtypes = [_P, _I64, _P, _P]
        for n in ("orc_q4k_block_ints", "orc_q5k_block_ints", "orc_q6k_block_ints"):
            getattr(L, n).argtypes = [_P, _P, _P, _P, _P]
        for n in ("orc_q4k_row_dot", "orc_q5k_row_dot", "orc_q6k_row_dot"):
            getattr(L, n).argtypes = [_I, _P, _P, _P, _P]
            getattr(L, n).restype = _F
        for n in ("orc_q8_0_row_dot", "orc_q8_0_row_dot_scalar"):
            getattr(L, n).argtypes = [_I64, _P, _P, _P]
            getattr(L, n).restype = _F
        L.orc_dequant_block.argtypes = [_I, _P, _P]
        L.orc_matmul.argtypes = [_I, _P, _I64, _I64, _P, _I64, _P, _P, _P, _P]
        L.orc_matmul.restype = _I
        L.orc_sample_with.argtypes = [_P, _I64, _P, _P, _P, _P, C.c_int32]
        L.orc_sample_with.restype = C.c_int32
        L.orc_chunked_step.argtypes = [_I, _I, _P, _P, _P, _P, _P, _P, _P]
        L.orc_chunked_step.restype = _I
        L.orc_libm_mismatches.argtypes = [_I, C.c_uint32, _I64, _P, C.POINTER(C.c_uint32)]
        L.orc_libm_mismatches.restype = _I64
        self.L = L

    def libm_mismatches(self, fn: int, first: int, vals: np.ndarray):
        """(count, first differing bit pattern or None) of vals[j] against the
        host expf (fn 0) / logf (fn 1) at bit pattern first + j."""
        vals = np.ascontiguousarray(vals, np.float32)
        bad = C.c_uint32(0)
        n = self.L.orc_libm_mismatches(fn, first, vals.size, vals.ctypes.data, C.byref(bad))
        return int(n), (int(bad.value) if n else None)

    def chunked_prefill(self, q, k, v, g_log, beta, state):
        """slm_forward_ssm_batch's chunk loop (slm/qwen.c:777-806) for one head:
        q, k, v [n][hd], g_log, beta [n]; state [hd][hd] is updated in place.
        Returns out [n][hd]."""
        return _chunked_loop(lambda *a: self.L.orc_chunked_step(*a), q, k, v, g_log, beta, state)

    def sample_with(self, logits: np.ndarray, sp: dict, st: np.ndarray, hist) -> int:
        """Restated sample_with on `logits` (float32, penalized in place) with
        the generator words `st` (uint64[2], advanced in place)."""
        assert logits.dtype == np.float32 and logits.flags.c_contiguous
        fp = np.array([sp["temperature"], sp["top_p"], sp["min_p"], sp["repetition_penalty"]], np.float32)
        ip = np.array([sp["top_k"], sp["repetition_window"]], np.int32)
        h = np.ascontiguousarray(hist, np.int32)
        return int(self.L.orc_sample_with(_ptr(logits), logits.size, _ptr(fp), _ptr(ip), _ptr(st),
                                          _ptr(h) if h.size else None, int(h.size)))

    def quantize_q8k(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, k = x.reshape(-1, x.shape[-1]).shape
        qs = np.empty((n, k), np.int8)
        d = np.empty((n, k // 256), np.float32)
        bs = np.empty((n, k // 256, 16), np.int16)
        for t in range(n):
            self.L.orc_quantize_row_q8k(_ptr(x.reshape(n, k)[t]), k, _ptr(d[t]), _ptr(qs[t]), _ptr(bs[t]))
        return qs, d, bs

    def quantize_q8_0(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, k = x.reshape(-1, x.shape[-1]).shape
        qs = np.empty((n, k), np.int8)
        d = np.empty((n, k // 32), np.uint16)
        for t in range(n):
            self.L.orc_quantize_row_q8_0(_ptr(x.reshape(n, k)[t]), k, _ptr(d[t]), _ptr(qs[t]))
        return qs, d

    def block_ints(self, gtype, blk: np.ndarray, q8: np.ndarray, bs: np.ndarray):
        fn = {Q4_K: self.L.orc_q4k_block_ints, Q5_K: self.L.orc_q5k_block_ints,
              Q6_K: self.L.orc_q6k_block_ints}[gtype]
        a, b = C.c_int32(), C.c_int32()
        blk = np.ascontiguousarray(blk, np.uint8)
        q8 = np.ascontiguousarray(q8, np.int8)
        bs = np.ascontiguousarray(bs, np.int16)
        fn(_ptr(blk), _ptr(q8), _ptr(bs), C.byref(a), C.byref(b))
        return a.value, b.value

    def matvec_preq(self, gtype, w: np.ndarray, out_f: int, k: int, qs, d, bs=None) -> np.ndarray:
        """Row dots of every weight row against ONE pre-quantized row."""
        out = np.empty(out_f, np.float32)
        rb = (k // BLOCK_WEIGHTS[gtype]) * BLOCK_BYTES[gtype]
        w = np.ascontiguousarray(w, np.uint8)
        qs = np.ascontiguousarray(qs, np.int8)
        d = np.ascontiguousarray(d)
        if gtype == Q8_0:
            for j in range(out_f):
                out[j] = self.L.orc_q8_0_row_dot(k, C.c_void_p(w.ctypes.data + j * rb), _ptr(d), _ptr(qs))
            return out
        bs = np.ascontiguousarray(bs, np.int16)
        fn = {Q4_K: self.L.orc_q4k_row_dot, Q5_K: self.L.orc_q5k_row_dot, Q6_K: self.L.orc_q6k_row_dot}[gtype]
        for j in range(out_f):
            out[j] = fn(k // 256, C.c_void_p(w.ctypes.data + j * rb), _ptr(d), _ptr(qs), _ptr(bs))
        return out

    def matmul(self, gtype, w: np.ndarray, out_f: int, k: int, x: np.ndarray) -> np.ndarray:
        """tensor_matmul_*_f32 restatement: x fp32 [n, k] -> out [n, out_f]."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
        n = x.shape[0]
        out = np.empty((n, out_f), np.float32)
        sq = np.empty(k, np.int8)
        sd = np.empty(max(k // 32, 1), np.float32)
        sb = np.empty(max(k // 16, 1), np.int16)
        w = np.ascontiguousarray(w, np.uint8)
        rc = self.L.orc_matmul(gtype, _ptr(w), out_f, k, _ptr(x), n, _ptr(out), _ptr(sq), _ptr(sd), _ptr(sb))
        if rc != 0:
            raise ValueError(f"orc_matmul rejected type {gtype} k {k}")
        return out

    def dequant_block(self, gtype, blk: np.ndarray) -> np.ndarray:
        y = np.empty(256, np.float32)
        self.L.orc_dequant_block(gtype, _ptr(np.ascontiguousarray(blk, np.uint8)), _ptr(y))
        return y


def _chunked_loop(step, q, k, v, g_log, beta, state):
    """Runs `step` (a chunked_ssm_step_f32 of <= 64 tokens) over the tokens in
    64-token chunks with the state carried, as slm_forward_ssm_batch does."""
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    g_log, beta = (np.ascontiguousarray(a, np.float32) for a in (g_log, beta))
    assert state.dtype == np.float32 and state.flags.c_contiguous
    n, hd = q.shape
    out = np.empty((n, hd), np.float32)
    for c0 in range(0, n, 64):
        cn = min(64, n - c0)
        o = np.empty((cn, hd), np.float32)
        sl = [np.ascontiguousarray(a[c0:c0 + cn]) for a in (q, k, v, g_log, beta)]
        rc = step(cn, hd, *[_ptr(a) for a in sl[:3]], _ptr(sl[3]), _ptr(sl[4]), _ptr(state), _ptr(o))
        assert rc == 0, "chunked step rejected its arguments"
        out[c0:c0 + cn] = o
    return out


class Ref:
    """The reference's own C code (oracle/_ref/libqhref.so)."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self):
        path = REF_SO
        if not os.path.exists(path):
            build(force=True)
        L = C.CDLL(path)
        L.ref_simd_init()
        L.ref_dispatch_label.restype = C.c_char_p
        for n in ("ref_q4k_row_dot", "ref_q5k_row_dot", "ref_q6k_row_dot",
                  "ref_scalar_q4k_row_dot", "ref_scalar_q5k_row_dot", "ref_scalar_q6k_row_dot"):
            getattr(L, n).argtypes = [_I, _P, _P]
            getattr(L, n).restype = _F
        for n in ("ref_q8_0_dot", "ref_scalar_q8_0_dot"):
            getattr(L, n).argtypes = [_P, _P, _I64]
            getattr(L, n).restype = _F
        L.ref_quantize_row_q8k.argtypes = [_P, _P, _I64]
        L.ref_quantize_row_q8_0.argtypes = [_P, _P, _I64]
        L.ref_dequant_block.argtypes = [_I, _P, _P]
        L.ref_matmul.argtypes = [_I, _P, _I64, _I64, _P, _I64, _P]
        L.ref_matmul.restype = _I
        L.ref_matvec_mt.argtypes = [_I, _P, _I64, _I64, _P, _P, _I]
        L.ref_matvec_mt.restype = _I
        L.ref_matvec_pool_mt.argtypes = [_I, _P, _I, _I64, _I64, _P, _P, _I]
        L.ref_matvec_pool_mt.restype = _I
        L.ref_sample_with.argtypes = [_P, _I64, _P, _P, _P, _P, C.c_int32]
        L.ref_sample_with.restype = C.c_int32
        L.ref_rng_seed.argtypes = [C.c_uint64, _P]
        L.ref_sampler_defaults.argtypes = [_P, _P]
        L.ref_chunked_step.argtypes = [C.c_int32] * 3 + [_P] * 7
        L.ref_chunked_step.restype = _I
        self.L = L
        self.label = L.ref_dispatch_label().decode()

    # -- sampler chain (slm/sampler.c:134-180, slm/model.c:414-447) --------
    def rng_seed(self, seed: int) -> np.ndarray:
        st = np.zeros(2, np.uint64)
        self.L.ref_rng_seed(seed, _ptr(st))
        return st

    def sampler_defaults(self):
        fp, ip = np.zeros(4, np.float32), np.zeros(2, np.int32)
        self.L.ref_sampler_defaults(_ptr(fp), _ptr(ip))
        return {"temperature": float(fp[0]), "top_p": float(fp[1]), "min_p": float(fp[2]),
                "repetition_penalty": float(fp[3]), "top_k": int(ip[0]), "repetition_window": int(ip[1])}

    def sample_with(self, logits: np.ndarray, sp: dict, st: np.ndarray, hist) -> int:
        """sample_with on `logits` (float32, modified in place) with the
        generator words `st` (uint64[2], advanced in place)."""
        assert logits.dtype == np.float32 and logits.flags.c_contiguous
        fp = np.array([sp["temperature"], sp["top_p"], sp["min_p"], sp["repetition_penalty"]], np.float32)
        ip = np.array([sp["top_k"], sp["repetition_window"]], np.int32)
        h = np.ascontiguousarray(hist, np.int32)
        return int(self.L.ref_sample_with(_ptr(logits), logits.size, _ptr(fp), _ptr(ip), _ptr(st),
                                          _ptr(h) if h.size else None, int(h.size)))

    def quantize_q8k(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
        n, k = x.shape
        raws = []
        for t in range(n):
            raw = np.empty((k // 256) * 292, np.uint8)
            self.L.ref_quantize_row_q8k(_ptr(x[t]), _ptr(raw), k)
            raws.append(raw)
        parts = [from_q8k_blocks(r, k) for r in raws]
        return (np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]),
                np.stack([p[2] for p in parts]))

    def quantize_q8_0(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
        n, k = x.shape
        parts = []
        for t in range(n):
            raw = np.empty((k // 32) * 34, np.uint8)
            self.L.ref_quantize_row_q8_0(_ptr(x[t]), _ptr(raw), k)
            parts.append(from_q8_0_blocks(raw, k))
        return np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts])

    def matmul(self, gtype, w: np.ndarray, out_f: int, k: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
        n = x.shape[0]
        out = np.empty((n, out_f), np.float32)
        w = np.ascontiguousarray(w, np.uint8)
        rc = self.L.ref_matmul(gtype, _ptr(w), out_f, k, _ptr(x), n, _ptr(out))
        if rc != 0:
            raise ValueError(f"ref_matmul rejected type {gtype}")
        return out

    def row_dot(self, gtype, row: np.ndarray, xq_blocks: np.ndarray, k: int, scalar=False) -> float:
        row = np.ascontiguousarray(row, np.uint8)
        if gtype == Q8_0:
            fn = self.L.ref_scalar_q8_0_dot if scalar else self.L.ref_q8_0_dot
            return fn(_ptr(row), _ptr(xq_blocks), k)
        name = {Q4_K: "q4k", Q5_K: "q5k", Q6_K: "q6k"}[gtype]
        fn = getattr(self.L, f"ref_scalar_{name}_row_dot" if scalar else f"ref_{name}_row_dot")
        return fn(k // 256, _ptr(row), _ptr(xq_blocks))

    def matvec_mt(self, gtype, w: np.ndarray, out_f: int, k: int, xq_blocks: np.ndarray,
                  nthreads: int, out: np.ndarray = None) -> np.ndarray:
        if out is None:
            out = np.empty(out_f, np.float32)
        self.L.ref_matvec_mt(gtype, _ptr(w), out_f, k, _ptr(xq_blocks), _ptr(out), nthreads)
        return out

    def matvec_pool_mt(self, gtype, pool, out_f: int, k: int, xq_blocks: np.ndarray,
                       nthreads: int, out: np.ndarray) -> None:
        """Every matrix of `pool` against one activation row, rows over threads."""
        ptrs = (C.c_void_p * len(pool))(*[w.ctypes.data for w in pool])
        self.L.ref_matvec_pool_mt(gtype, ptrs, len(pool), out_f, k, _ptr(xq_blocks), _ptr(out), nthreads)

    def chunked_prefill(self, q, k, v, g_log, beta, state):
        """The reference's own chunked_ssm_step_f32 in slm_forward_ssm_batch's
        chunk loop; same arguments as Oracle.chunked_prefill."""
        return _chunked_loop(lambda n, hd, *a: self.L.ref_chunked_step(n, hd, hd, *a), q, k, v, g_log, beta, state)

    def dequant_block(self, gtype, blk: np.ndarray) -> np.ndarray:
        y = np.empty(256, np.float32)
        self.L.ref_dequant_block(gtype, _ptr(np.ascontiguousarray(blk, np.uint8)), _ptr(y))
        return y


class RefModel:
    """The reference's slm_forward_step over a synthetic blob's tensors, or
    over a GGUF file read by the reference's own loader (RefModel.from_gguf:
    gguf_open slm/gguf.c:172, slm_load_config slm/qwen.c:59,
    slm_load_weights slm/qwen.c:174)."""

    @staticmethod
    def _bind(L):
        L.ref_model_create.restype = C.c_void_p
        L.ref_model_create.argtypes = [_P, _P, _I, _P, _P, _P, _P]
        L.ref_model_from_gguf.restype = C.c_void_p
        L.ref_model_from_gguf.argtypes = [C.c_char_p, _P, _P]
        L.ref_model_step.argtypes = [_P, C.c_int32, C.c_int32, _P]
        L.ref_model_step.restype = C.c_int
        L.ref_model_destroy.argtypes = [_P]
        L.ref_model_snapshot.argtypes = [_P, C.c_int32]
        L.ref_model_snapshot.restype = C.c_void_p
        L.ref_model_restore.argtypes = [_P, _P]
        L.ref_snapshot_free.argtypes = [_P]
        L.ref_trace_begin.argtypes = [C.c_char_p]
        L.ref_trace_begin.restype = C.c_int
        L.ref_model_forward_batch.argtypes = [_P, _P, C.c_int32, C.c_int32, _P]
        L.ref_model_forward_batch.restype = C.c_int

    @classmethod
    def from_gguf(cls, ref: "Ref", path: str):
        """Returns (model, ic[17], fc[2]): the reference's config as read
        from the file (ic: layers, hidden, ffn, vocab, heads, kv heads,
        head dim, rope dim, sections[4], gdn heads, gdn head dim, conv,
        full-attention interval, max position; fc: rope theta, eps)."""
        cls._bind(ref.L)
        ic, fc = np.zeros(17, np.int32), np.zeros(2, np.float32)
        h = ref.L.ref_model_from_gguf(path.encode(), _ptr(ic), _ptr(fc))
        if not h:
            raise RuntimeError(f"reference gguf load failed: {path}")
        m = cls.__new__(cls)
        m.L, m.vocab, m.h, m._keep = ref.L, int(ic[3]), h, ()
        return m, ic, fc

    def __init__(self, ref: "Ref", cfg, tensors):
        L = ref.L
        self._bind(L)
        ic = np.array([cfg.n_layers, cfg.hidden, cfg.ffn, cfg.vocab, cfg.n_heads, cfg.n_kv_heads,
                       cfg.head_dim, cfg.rope_dim, *list(cfg.rope_sections), cfg.gdn_heads,
                       cfg.gdn_head_dim, cfg.conv_kernel, cfg.full_attn_interval, cfg.max_pos], np.int32)
        fc = np.array([cfg.rope_theta, cfg.norm_eps], np.float32)
        n = len(tensors)
        self._names = [t[0].encode() for t in tensors]
        names = (C.c_char_p * n)(*self._names)
        types = np.array([t[1] for t in tensors], np.int32)
        shapes = np.array([t[2] for t in tensors], np.int64).reshape(n, 2)
        datas = (C.c_void_p * n)(*[t[3] for t in tensors])
        self._keep = (ic, fc, names, types, shapes, datas)
        self.L, self.vocab = L, cfg.vocab
        self.h = L.ref_model_create(_ptr(ic), _ptr(fc), n, names, _ptr(types), _ptr(shapes), datas)

    def step(self, tok: int, pos: int, want_logits: bool = False):
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        a = self.L.ref_model_step(self.h, int(tok), int(pos), _ptr(logits) if logits is not None else None)
        return (a, logits) if want_logits else a

    def forward_batch(self, toks, pos_start: int, want_logits: bool = False):
        """slm_forward_batch (the LLM_USE_FORWARD_BATCH prefill) over `toks` at
        positions pos_start..; returns the last token's argmax (and logits)."""
        t = np.ascontiguousarray(toks, np.int32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        a = self.L.ref_model_forward_batch(self.h, _ptr(t), len(t), int(pos_start),
                                           _ptr(logits) if logits is not None else None)
        return (a, logits) if want_logits else a

    def snapshot(self, pos: int):
        """slm_ctx_snapshot at position pos; free with free_snapshot."""
        return self.L.ref_model_snapshot(self.h, pos)

    def restore(self, snap):
        self.L.ref_model_restore(self.h, snap)

    def free_snapshot(self, snap):
        self.L.ref_snapshot_free(snap)

    def trace_step(self, path: str, tok: int, pos: int):
        """One slm_forward_step with the reference's JSONL tracer writing to path."""
        if self.L.ref_trace_begin(path.encode()) != 0:
            raise RuntimeError(f"cannot open {path}")
        try:
            return self.step(tok, pos)
        finally:
            self.L.ref_trace_end()

    def close(self):
        if self.h:
            self.L.ref_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
