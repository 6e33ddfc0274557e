# SPDX-License-Identifier: MIT
"""Host-side mirror of the reference's matmul interface over libqh200.

``matmul(gtype, w, k, out_f, x)`` is matmul_dispatch (slm/model.c:220) and
``tensor_matmul_q4k_f32(w, out_f, k, x)`` etc. mirror slm/tensor.c:827-1033:
same argument meaning, x is fp32 [n_tok, k], the result is fp32
[n_tok, out_f]. Device memory comes from torch CUDA tensors (plumbing only);
every computation is a libqh200 kernel launched on torch's current stream.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import (BLOCK_BYTES, BLOCK_WEIGHTS, MatvecJob, Q4_K, Q5_K, Q6_K, Q8_0, QHError, check,
               lib)

# ---------------------------------------------------------------------------
# Synthetic inputs (host only, no GPU needed)
# ---------------------------------------------------------------------------


def synth_blocks(gtype: int, n_blocks: int, seed: int) -> np.ndarray:
    out = np.empty(n_blocks * BLOCK_BYTES[gtype], dtype=np.uint8)
    check(lib().qh_synth_blocks(gtype, n_blocks, seed, out.ctypes.data), "qh_synth_blocks")
    return out


def synth_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    check(lib().qh_synth_normal(seed, n, mean, std, out.ctypes.data), "qh_synth_normal")
    return out


def synth_quantize(gtype: int, w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    out = np.empty(rows * (k // BLOCK_WEIGHTS[gtype]) * BLOCK_BYTES[gtype], dtype=np.uint8)
    check(lib().qh_synth_quantize(gtype, w.ctypes.data, rows, k, out.ctypes.data), "qh_synth_quantize")
    return out


# ---------------------------------------------------------------------------
# Device plumbing (torch tensors as allocations, torch's stream as the stream)
# ---------------------------------------------------------------------------


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise QHError(-3, "device", "no CUDA device visible; the qh200 kernels need a B200")
    return torch


def stream_handle():
    return C.c_void_p(_torch().cuda.current_stream().cuda_stream)


def to_device(a: np.ndarray):
    torch = _torch()
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda")
    return t


def dptr(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def quantize_q8k(x, k: int, n_tok: int):
    """qh_quantize_q8k into a fresh split buffer (uint8 tensor)."""
    torch = _torch()
    buf = torch.zeros(int(lib().qh_q8k_bytes(k, n_tok)), dtype=torch.uint8, device="cuda")
    check(lib().qh_quantize_q8k(dptr(x), k, n_tok, dptr(buf), stream_handle()), "qh_quantize_q8k")
    return buf


def quantize_q8_0(x, k: int, n_tok: int):
    torch = _torch()
    buf = torch.zeros(int(lib().qh_q8_0_bytes(k, n_tok)), dtype=torch.uint8, device="cuda")
    check(lib().qh_quantize_q8_0(dptr(x), k, n_tok, dptr(buf), stream_handle()), "qh_quantize_q8_0")
    return buf


def unpack_q8k(buf: np.ndarray, k: int, n_tok: int):
    """(qs int8 [n_tok,k], d f32 [n_tok,k/256], bsums int16 [n_tok,k/256,16])."""
    L = lib()
    nb = k // 256
    stride = (nb + 3) // 4 * 4          # scale rows padded to 16 bytes
    d_off, b_off = int(L.qh_q8k_d_offset(k, n_tok)), int(L.qh_q8k_bsums_offset(k, n_tok))
    qs = buf[: k * n_tok].view(np.int8).reshape(n_tok, k)
    d = buf[d_off: d_off + 4 * stride * n_tok].view(np.float32).reshape(n_tok, stride)[:, :nb]
    bs = buf[b_off: b_off + 32 * nb * n_tok].view(np.int16).reshape(n_tok, nb, 16)
    return qs, d, bs


def unpack_q8_0(buf: np.ndarray, k: int, n_tok: int):
    """(qs int8 [n_tok,k], d fp16 bits uint16 [n_tok,k/32])."""
    nb = k // 32
    stride = (nb + 7) // 8 * 8          # scale rows padded to 16 bytes
    d_off = int(lib().qh_q8_0_d_offset(k, n_tok))
    qs = buf[: k * n_tok].view(np.int8).reshape(n_tok, k)
    d = buf[d_off: d_off + 2 * stride * n_tok].view(np.uint16).reshape(n_tok, stride)[:, :nb]
    return qs, d


def matmul(gtype: int, w, k: int, out_f: int, x, n_tok: int = None, out=None, work=None):
    """matmul_dispatch mirror: w device GGUF blocks (k, out_f), x fp32 [n_tok, k]."""
    torch = _torch()
    if n_tok is None:
        n_tok = x.numel() // k
    if out is None:
        out = torch.empty((n_tok, out_f), dtype=torch.float32, device="cuda")
    need = int(lib().qh_matmul_workspace_bytes(gtype, k, n_tok))
    if need < 0:
        raise QHError(-2, "matmul", f"unsupported type {gtype}")
    if work is None or work.numel() < need:
        work = torch.empty(need, dtype=torch.uint8, device="cuda")
    check(lib().qh_matmul(gtype, dptr(w), k, out_f, dptr(x), n_tok, dptr(out), dptr(work),
                          work.numel(), stream_handle()), "qh_matmul")
    return out


def matmul_gemm(gtype: int, w, k: int, out_f: int, x, n_tok: int = None, out=None):
    """Tensor-core path of matmul (qh_matmul_gemm): same results, many tokens."""
    torch = _torch()
    if n_tok is None:
        n_tok = x.numel() // k
    if out is None:
        out = torch.empty((n_tok, out_f), dtype=torch.float32, device="cuda")
    need = int(lib().qh_matmul_gemm_workspace_bytes(gtype, k, out_f, n_tok))
    if need < 0:
        raise QHError(-2, "matmul_gemm", f"unsupported type {gtype} or shape")
    work = torch.empty(need, dtype=torch.uint8, device="cuda")
    check(lib().qh_matmul_gemm(gtype, dptr(w), k, out_f, dptr(x), n_tok, dptr(out), dptr(work), need, None),
          "qh_matmul_gemm")
    return out


def gemm_pack(gtype: int, w, k: int, out_f: int):
    """qh_gemm_pack_weights into a fresh device buffer."""
    torch = _torch()
    wt = torch.empty(int(lib().qh_gemm_weight_bytes(gtype, k, out_f)), dtype=torch.uint8, device="cuda")
    check(lib().qh_gemm_pack_weights(gtype, dptr(w), k, out_f, dptr(wt), None), "qh_gemm_pack_weights")
    return wt


def gemm_expand(gtype: int, wt, k: int, out_f: int):
    """qh_gemm_expand_weights of tiled weights into a fresh device buffer
    (use with qh_gemm flags QH_GEMM_EXPANDED)."""
    torch = _torch()
    we = torch.empty(int(lib().qh_gemm_expanded_bytes(gtype, k, out_f)), dtype=torch.uint8, device="cuda")
    check(lib().qh_gemm_expand_weights(gtype, dptr(wt), k, out_f, dptr(we), None), "qh_gemm_expand_weights")
    return we


def quantize_q8kt(x, k: int, n_tok: int):
    torch = _torch()
    buf = torch.empty(int(lib().qh_q8kt_bytes(k, n_tok)), dtype=torch.uint8, device="cuda")
    check(lib().qh_quantize_q8kt(dptr(x), k, n_tok, dptr(buf), None), "qh_quantize_q8kt")
    return buf


def gemm(gtype: int, jobs, k: int, xq, n_tok: int, split: bool = True, flags: int = 0):
    """qh_gemm over jobs [(wt, out_f, out, ld_out)] sharing tiled activations xq;
    split=True passes a fresh zeroed scratch so small launches may split K."""
    from . import GemmJob
    torch = _torch()
    arr = (GemmJob * len(jobs))(*[GemmJob(wt.data_ptr(), out_f, out.data_ptr(), ld) for wt, out_f, out, ld in jobs])
    scratch, nbytes = None, 0
    if split:
        nbytes = int(lib().qh_gemm_scratch_bytes(C.cast(arr, C.c_void_p), len(jobs), k, n_tok))
        scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    check(lib().qh_gemm(gtype, C.cast(arr, C.c_void_p), len(jobs), k, dptr(xq), n_tok,
                        dptr(scratch) if scratch is not None else None, nbytes, flags, None), "qh_gemm")
    return scratch


def tensor_matmul_q4k_f32(w, out_f, k, x):
    return matmul(Q4_K, w, k, out_f, x)


def tensor_matmul_q5k_f32(w, out_f, k, x):
    return matmul(Q5_K, w, k, out_f, x)


def tensor_matmul_q6k_f32(w, out_f, k, x):
    return matmul(Q6_K, w, k, out_f, x)


def tensor_matmul_q8_0_f32(w, out_f, k, x):
    return matmul(Q8_0, w, k, out_f, x)


class MatvecPlan:
    """Grouped matvec plan over device buffers.

    jobs = [(w, xq, out, k, out_f)] or [(w, xq, out, k, out_f, xq_rows, xq_row0)]
    where xq is a split activation buffer quantized for xq_rows rows and the
    job uses rows [xq_row0, xq_row0 + n_tok).
    """

    def __init__(self, gtype: int, jobs, n_tok: int = 1):
        arr = (MatvecJob * len(jobs))()
        for i, job in enumerate(jobs):
            w, xq, out, k, out_f = job[:5]
            rows, row0 = (job[5], job[6]) if len(job) > 5 else (0, 0)
            arr[i] = MatvecJob(w.data_ptr(), xq.data_ptr(), out.data_ptr(), k, out_f, rows, row0)
        self._keep = jobs
        h = C.c_void_p()
        check(lib().qh_matvec_plan_create(gtype, arr, len(jobs), n_tok, C.byref(h)),
              "qh_matvec_plan_create")
        self.handle = h

    def run(self, stream=None):
        check(lib().qh_matvec_plan_run(self.handle, stream if stream is not None else stream_handle()),
              "qh_matvec_plan_run")

    def fuse_input(self, mode: int, a=None, b=None, w=None, eps: float = 0.0, h_out=None):
        """qh_matvec_plan_fuse_input (QH_FUSE_RMSNORM 1, SWIGLU 2, QUANT 3; 0 = off)."""
        self._fused = (a, b, w, h_out)
        check(lib().qh_matvec_plan_fuse_input(self.handle, mode, *(dptr(t) if t is not None else None
                                                                  for t in (a, b, w)),
                                              eps, dptr(h_out) if h_out is not None else None),
              "qh_matvec_plan_fuse_input")

    def fuse_output(self, mode: int, k: int, xq, a=None, b=None, w=None, eps: float = 0.0, h_out=None):
        """qh_matvec_plan_fuse_output: the launch's last CTA forms the Q8_K rows
        xq (split layout) from a/b (same modes as fuse_input; 0 = off)."""
        self._tail = (xq, a, b, w, h_out)
        check(lib().qh_matvec_plan_fuse_output(self.handle, mode, k, *(dptr(t) if t is not None else None
                                                                       for t in (a, b, w)),
                                               eps, dptr(h_out) if h_out is not None else None,
                                               dptr(xq) if xq is not None else None),
              "qh_matvec_plan_fuse_output")

    def info(self):
        r, s, g, m = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        check(lib().qh_matvec_plan_info(self.handle, C.byref(r), C.byref(s), C.byref(g), C.byref(m)),
              "qh_matvec_plan_info")
        return {"rows_per_tile": r.value, "stages": s.value, "grid": g.value, "smem": m.value}

    def close(self):
        if self.handle:
            lib().qh_matvec_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# Model level (include/qh_slm.h)
# ---------------------------------------------------------------------------
from . import SlmConfig  # noqa: E402


def slm_config(max_pos: int = 320, **over) -> SlmConfig:
    """BASELINE config 4 shape (qh_slm_config_default) with field overrides."""
    c = SlmConfig()
    lib().qh_slm_config_default(C.byref(c), max_pos)
    for k, v in over.items():
        if k == "rope_sections":
            for i, x in enumerate(v):
                c.rope_sections[i] = x
        else:
            setattr(c, k, v)
    return c


class Blob:
    """Weight blob: synthetic (qh_blob_synthetic) or read from a GGUF file
    (Blob.from_gguf, qh_gguf_load)."""

    def __init__(self, cfg: SlmConfig, seed: int = None, handle=None, mix: int = 0):
        """mix: 0 BASELINE types, 1 the released Q4_K_M file's types, 2 every type (qh_blob_synthetic_mix)."""
        if handle is None:
            h = C.c_void_p()
            check(lib().qh_blob_synthetic_mix(C.byref(cfg), seed, mix, C.byref(h)), "qh_blob_synthetic_mix")
            handle = h
        self.handle, self.cfg = handle, cfg

    @classmethod
    def empty(cls, cfg: SlmConfig):
        """An empty blob to fill with add() (qh_blob_create)."""
        h = C.c_void_p()
        check(lib().qh_blob_create(C.byref(h)), "qh_blob_create")
        return cls(cfg, handle=h)

    def add(self, name: str, gtype: int, shape, data: bytes):
        """qh_blob_add: copies the tensor's bytes."""
        sh = (C.c_int64 * 2)(*shape)
        check(lib().qh_blob_add(self.handle, name.encode(), gtype, sh, data, len(data)), "qh_blob_add")

    @classmethod
    def from_gguf(cls, path: str, max_pos_cap: int = 0):
        cfg, h = SlmConfig(), C.c_void_p()
        check(lib().qh_gguf_load(path.encode(), max_pos_cap, C.byref(cfg), C.byref(h)), "qh_gguf_load")
        return cls(cfg, handle=h)

    def write_gguf(self, path: str, cfg: SlmConfig = None):
        check(lib().qh_gguf_write(path.encode(), C.byref(cfg or self.cfg), self.handle), "qh_gguf_write")

    def tensors(self):
        """[(name, type, (shape0, shape1), data pointer, nbytes)]"""
        L, out = lib(), []
        for i in range(L.qh_blob_count(self.handle)):
            name, typ, data, nb = C.c_char_p(), C.c_int32(), C.c_void_p(), C.c_int64()
            shape = (C.c_int64 * 2)()
            check(L.qh_blob_tensor(self.handle, i, C.byref(name), C.byref(typ), shape, C.byref(data),
                                   C.byref(nb)), "qh_blob_tensor")
            out.append((name.value.decode(), typ.value, (shape[0], shape[1]), data.value, nb.value))
        return out

    def close(self):
        if self.handle:
            lib().qh_blob_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sampler_defaults():
    """qh_sampler_defaults (slm_sampler_defaults)."""
    from . import Sampler
    sp = Sampler()
    lib().qh_sampler_defaults(C.byref(sp))
    return sp


def rng_seed(seed: int) -> np.ndarray:
    """qh_rng_seed: the generator's two words for `seed`."""
    st = np.zeros(2, np.uint64)
    lib().qh_rng_seed(seed, st.ctypes.data)
    return st


def sample(sp, logits, hist, hist_n, rng):
    """qh_sample on device tensors: logits float32 [B][vocab] (penalized in
    place), hist int32 [B][stride], hist_n int32 [B], rng uint64-as-int64
    [B][2] (advanced in place). Returns the int32 [B] picks (device)."""
    torch = _torch()
    B, vocab = logits.shape
    out = torch.empty(B, dtype=torch.int32, device=logits.device)
    check(lib().qh_sample(C.byref(sp), dptr(logits), B, vocab, dptr(hist), hist.shape[1], dptr(hist_n), dptr(rng),
                          dptr(out), stream_handle()), "qh_sample")
    return out


class Snapshot:
    """A qh_slm_snap (device memory), freed with the object."""

    def __init__(self, handle):
        self.handle = handle

    @property
    def nbytes(self) -> int:
        return int(lib().qh_slm_snapshot_bytes(self.handle))

    @property
    def pos(self) -> int:
        return int(lib().qh_slm_snapshot_pos(self.handle))

    def close(self):
        if self.handle:
            lib().qh_slm_snapshot_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Slm:
    """Device model with n_seq sequences (qh_slm_create)."""

    def __init__(self, cfg: SlmConfig, blob: Blob, n_seq: int = 1):
        _torch()
        h = C.c_void_p()
        check(lib().qh_slm_create(C.byref(cfg), blob.handle, n_seq, C.byref(h)), "qh_slm_create")
        self.handle, self.cfg, self.n_seq = h, cfg, n_seq

    def reset(self):
        check(lib().qh_slm_reset(self.handle), "qh_slm_reset")

    def step(self, tokens, pos: int, want_logits: bool = False):
        toks = np.ascontiguousarray(tokens, np.int32).reshape(self.n_seq)
        nxt = np.empty(self.n_seq, np.int32)
        logits = np.empty((self.n_seq, self.cfg.vocab), np.float32) if want_logits else None
        check(lib().qh_slm_step(self.handle, toks.ctypes.data, pos, nxt.ctypes.data,
                                logits.ctypes.data if logits is not None else None), "qh_slm_step")
        return (nxt, logits) if want_logits else nxt

    def generate(self, prompt, n_new: int):
        p = np.ascontiguousarray(prompt, np.int32).reshape(self.n_seq, -1)
        out = np.empty((self.n_seq, n_new), np.int32)
        check(lib().qh_slm_generate(self.handle, p.ctypes.data, p.shape[1], n_new, out.ctypes.data),
              "qh_slm_generate")
        return out

    def generate_sampled(self, prompt, max_new: int, sampler=None, seeds=None, min_new: int = 0,
                         eos_id: int = -1, eot_id: int = -1, stop_ids=()):
        """qh_slm_generate_sampled: returns a list of n_seq int32 arrays
        (each sequence's tokens up to and including its first stop)."""
        p = np.ascontiguousarray(prompt, np.int32).reshape(self.n_seq, -1)
        sp = sampler if sampler is not None else sampler_defaults()
        sd = None if seeds is None else np.ascontiguousarray(seeds, np.uint64).reshape(self.n_seq)
        st = np.ascontiguousarray(list(stop_ids), np.int32)
        out = np.zeros((self.n_seq, max(max_new, 1)), np.int32)
        n_out = np.zeros(self.n_seq, np.int32)
        check(lib().qh_slm_generate_sampled(self.handle, p.ctypes.data, p.shape[1], max_new, min_new, C.byref(sp),
                                            sd.ctypes.data if sd is not None else None, eos_id, eot_id,
                                            st.ctypes.data if st.size else None, int(st.size), out.ctypes.data,
                                            n_out.ctypes.data), "qh_slm_generate_sampled")
        return [out[b, :n_out[b]].copy() for b in range(self.n_seq)]

    def trace(self, seq: int, path: str):
        """qh_slm_trace: the next step writes sequence seq's JSONL trace to path."""
        check(lib().qh_slm_trace(self.handle, seq, path.encode()), "qh_slm_trace")

    def snapshot(self) -> "Snapshot":
        """qh_slm_snapshot: the decode state of every sequence."""
        s = C.c_void_p()
        check(lib().qh_slm_snapshot(self.handle, C.byref(s)), "qh_slm_snapshot")
        return Snapshot(s)

    def restore(self, snap: "Snapshot"):
        check(lib().qh_slm_restore(self.handle, snap.handle), "qh_slm_restore")

    def begin(self, prompt):
        p = np.ascontiguousarray(prompt, np.int32).reshape(self.n_seq, -1)
        check(lib().qh_slm_begin(self.handle, p.ctypes.data, p.shape[1]), "qh_slm_begin")

    def prefill(self, prompt, chunk: int = 0, mode: int = None):
        """qh_slm_prefill; chunk and mode (PREFILL_STEPWISE / PREFILL_CHUNKED)
        apply from the first call on."""
        p = np.ascontiguousarray(prompt, np.int32).reshape(self.n_seq, -1)
        if chunk:
            check(lib().qh_slm_set_prefill_chunk(self.handle, chunk), "qh_slm_set_prefill_chunk")
        if mode is not None:
            check(lib().qh_slm_set_prefill_mode(self.handle, mode), "qh_slm_set_prefill_mode")
        check(lib().qh_slm_prefill(self.handle, p.ctypes.data, p.shape[1]), "qh_slm_prefill")

    def set_decode_mode(self, mode: int):
        """qh_slm_set_decode_mode (DECODE_PERSISTENT / DECODE_LAUNCHES)."""
        check(lib().qh_slm_set_decode_mode(self.handle, mode), "qh_slm_set_decode_mode")

    def decode_mode(self) -> int:
        """qh_slm_decode_mode: the form decode steps actually run."""
        return int(lib().qh_slm_decode_mode(self.handle))

    def advance(self, n_steps: int):
        check(lib().qh_slm_advance(self.handle, n_steps), "qh_slm_advance")

    def picks(self, from_pos: int, n: int):
        out = np.empty((self.n_seq, n), np.int32)
        check(lib().qh_slm_picks(self.handle, from_pos, n, out.ctypes.data), "qh_slm_picks")
        return out

    @property
    def stream(self) -> int:
        return lib().qh_slm_stream(self.handle) or 0

    @property
    def device_next(self) -> int:
        return lib().qh_slm_device_next(self.handle) or 0

    def close(self):
        if self.handle:
            lib().qh_slm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DataParallel:
    """qh_dp (include/qh_dp.h): the NCCL communicator of one rank of a
    data-parallel job -- the token gather after each decode step and the
    max-over-ranks of timings. The 128-byte unique id travels from rank 0 to
    the others through `exchange(id_bytes_or_None) -> id_bytes` (e.g. a
    torch.distributed broadcast, a file)."""

    def __init__(self, rank: int, world: int, exchange, timeout_ms: int = 0):
        L = lib()
        buf = (C.c_uint8 * 128)()
        if rank == 0:
            check(L.qh_dp_unique_id(buf), "qh_dp_unique_id")
        uid = exchange(bytes(buf) if rank == 0 else None)
        C.memmove(buf, uid, 128)
        h = C.c_void_p()
        check(L.qh_dp_create(buf, world, rank, timeout_ms, C.byref(h)), "qh_dp_create")
        self.handle, self.rank, self.world = h, rank, world

    @classmethod
    def from_torch(cls, dist, timeout_ms: int = 0):
        """The id broadcast over an initialized torch.distributed group."""
        def exchange(b):
            obj = [b]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]
        return cls(dist.get_rank(), dist.get_world_size(), exchange, timeout_ms)

    def gather(self, d_local: int, n: int, d_all: int, stream: int = 0):
        check(lib().qh_dp_gather_tokens(self.handle, C.c_void_p(d_local), n, C.c_void_p(d_all),
                                        C.c_void_p(stream) if stream else None), "qh_dp_gather_tokens")

    def wait(self, stream: int = 0):
        check(lib().qh_dp_wait(self.handle, C.c_void_p(stream) if stream else None), "qh_dp_wait")

    def max(self, values):
        v = (C.c_double * len(values))(*values)
        check(lib().qh_dp_max_f64(self.handle, v, len(values)), "qh_dp_max_f64")
        return list(v)

    def close(self):
        if self.handle:
            lib().qh_dp_destroy(self.handle)
            self.handle = None
