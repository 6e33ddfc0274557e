# SPDX-License-Identifier: MIT
"""The reference's slm.h entry points (include/slm.h) over the device model:
slm_model_load of a GGUF, slm_ctx_create, two conversation turns through
slm_generate_ids (the token-level loop of slm_generate_raw, slm/slm.c:
237-361) with the context continuing at its position, snapshot / restore,
stats. Compared token for token with the same loop run on the reference's
own slm_forward_step and sample_with (oracle/_ref), continuing positions and
generator across turns as the reference's context does.
"""
import ctypes as C

import numpy as np
import pytest

MIX = 1  # the released Q4_K_M file's weight types


@pytest.fixture(scope="module")
def gguf(qh, tmp_path_factory):
    cfg = qh.host.slm_config(64, n_layers=4, vocab=2048)
    blob = qh.host.Blob(cfg, 0x51A7, mix=MIX)
    path = str(tmp_path_factory.mktemp("slm") / "model.gguf")
    blob.write_gguf(path)
    return cfg, blob, path


def test_model_load_failure_is_reported(qh):
    L = qh.lib()
    m = L.slm_model_load(b"/nonexistent/model.gguf")
    assert m  # non-NULL even on failure, as the reference's
    assert not L.slm_model_loaded(m)
    assert b"cannot load" in L.slm_model_error(m)
    assert not L.slm_ctx_create(m)
    L.slm_model_unload(m)


def test_defaults_match_reference(qh, ref):
    d = qh.lib().slm_sampler_defaults()
    r = ref.sampler_defaults()
    for f in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty", "repetition_window"):
        assert np.float32(getattr(d, f)) == np.float32(r[f]), f
    c = qh.lib().slm_ctrl_defaults()
    assert (c.tools, c.think, c.effort, c.debug, c.trace_tokens, c.dump_layer) == (True, False, None, 1, False, -1)


class RefConversation:
    """slm_generate_raw's loop on the reference's slm_forward_step and
    sample_with, positions and generator carried across calls."""

    def __init__(self, ref, cfg, tensors, eos, eot, stops, bos=0):
        from oracle.oracle import RefModel
        self.ref, self.cfg = ref, cfg
        self.rm = RefModel(ref, cfg, tensors)
        self.pos, self.st = 0, ref.rng_seed(1)
        self.eos, self.eot, self.stops, self.bos = eos, eot, set(stops), bos

    def generate(self, prompt, max_new, min_new, sp, seed, stop_after=None):
        if seed:
            self.st = self.ref.rng_seed(seed)
        for t in prompt:
            self.rm.step(int(t), self.pos)
            self.pos += 1
        hist, out = [int(t) for t in prompt], []
        last = int(prompt[-1]) if len(prompt) else self.bos
        while len(out) < max_new and self.pos < self.cfg.max_pos:
            _, lg = self.rm.step(last, self.pos, want_logits=True)
            if len(out) < min_new:
                for t in (self.eos, self.eot):
                    if 0 <= t < self.cfg.vocab:
                        lg[t] = -np.inf
            nxt = self.ref.sample_with(lg, sp, self.st, np.array(hist, np.int32))
            hist.append(nxt)
            out.append(nxt)
            self.pos += 1
            if nxt in (self.eos, self.eot) or nxt in self.stops:
                break
            if stop_after is not None and len(out) >= stop_after:
                break
            last = nxt
        return out

    def close(self):
        self.rm.close()


def _generate(qh, ctx, prompt, max_new, min_new, sampler, seed, stop_after=None):
    L = qh.lib()
    seen = []

    def on_token(tok, user):
        seen.append(int(tok))
        return 1 if stop_after is not None and len(seen) >= stop_after else 0

    cb = qh.SLM_TOKEN_FN(on_token)
    p = np.ascontiguousarray(prompt, np.int32)
    sp = C.byref(sampler) if sampler is not None else None
    n = L.slm_generate_ids(ctx, p.ctypes.data if p.size else None, int(p.size), max_new, min_new, sp, seed, cb, None)
    assert n >= 0, "slm_generate_ids failed"
    toks, cnt = L.slm_ctx_tokens(ctx, C.byref(C.c_int32())), C.c_int32()
    L.slm_ctx_tokens(ctx, C.byref(cnt))
    return n, [toks[i] for i in range(cnt.value)], seen


def _sampler_dict(s):
    return {f: getattr(s, f) for f in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty",
                                       "repetition_window")}


@pytest.mark.gpu
@pytest.mark.parametrize("greedy", [False, True], ids=["sampled", "greedy"])
def test_two_turns_match_reference(qh, cuda, ref, gguf, greedy):
    """Turn 1 from position 0 with a seed, turn 2 continuing at the
    context's position with the generator carried over (seed 0): both turns
    equal the reference's loop token for token; slm_ctx_tokens holds every
    prompt and generated id in order; the stats are set."""
    cfg, blob, path = gguf
    L = qh.lib()
    model = L.slm_model_load(path.encode())
    assert L.slm_model_loaded(model), L.slm_model_error(model)
    ctx = L.slm_ctx_create(model)
    assert ctx
    assert L.slm_vocab_size(ctx) == cfg.vocab
    sampler = None if greedy else L.slm_sampler_defaults()
    sp = {f: 0 for f in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty", "repetition_window")} \
        if greedy else _sampler_dict(sampler)
    eos, bos = L.slm_eos_id(ctx), L.slm_bos_id(ctx)
    rc = RefConversation(ref, cfg, blob.tensors(), eos, -1, [], bos)
    rng = np.random.default_rng(5)
    p1 = rng.integers(1, cfg.vocab, 9).astype(np.int32)
    p2 = rng.integers(1, cfg.vocab, 5).astype(np.int32)
    n1, toks1, seen1 = _generate(qh, ctx, p1, 12, 3, sampler, 7)
    want1 = rc.generate(p1, 12, 3, sp, 7)
    assert toks1[len(p1):] == want1, "turn 1 differs from the reference"
    assert n1 == len(want1) and seen1 == [t for t in want1 if t != eos]
    assert L.slm_n_prefill(ctx) == len(p1) and L.slm_n_generated(ctx) == n1
    assert L.slm_pp_per_sec(ctx) > 0 and L.slm_tg_per_sec(ctx) > 0
    n2, toks2, _ = _generate(qh, ctx, p2, 10, 0, sampler, 0)
    want2 = rc.generate(p2, 10, 0, sp, 0)
    assert toks2 == list(p1) + want1 + list(p2) + want2, "turn 2 differs from the reference"
    rc.close()
    L.slm_ctx_destroy(ctx)
    L.slm_model_unload(model)


@pytest.mark.gpu
def test_snapshot_restore_and_callback_stop(qh, cuda, gguf):
    """A snapshot after turn 1, restored after turn 2, replays turn 2 to the
    same tokens (generator included); a callback that returns non-zero ends
    the turn after that token."""
    cfg, _, path = gguf
    L = qh.lib()
    model = L.slm_model_load(path.encode())
    ctx = L.slm_ctx_create(model)
    sampler = L.slm_sampler_defaults()
    rng = np.random.default_rng(9)
    p1 = rng.integers(1, cfg.vocab, 7).astype(np.int32)
    p2 = rng.integers(1, cfg.vocab, 4).astype(np.int32)
    _generate(qh, ctx, p1, 8, 8, sampler, 11)
    snap = L.slm_ctx_snapshot(ctx)
    assert snap
    n_a, toks_a, _ = _generate(qh, ctx, p2, 9, 9, sampler, 0)
    L.slm_ctx_restore(ctx, snap)
    n_b, toks_b, _ = _generate(qh, ctx, p2, 9, 9, sampler, 0)
    assert (n_a, toks_a) == (n_b, toks_b)
    L.slm_ctx_restore(ctx, snap)
    n_c, toks_c, seen = _generate(qh, ctx, p2, 9, 9, sampler, 0, stop_after=3)
    assert n_c == 3 and seen == toks_a[-n_a:][:3] and toks_c == toks_a[:len(toks_a) - n_a + 3]
    L.slm_snapshot_free(snap)
    L.slm_ctx_destroy(ctx)
    L.slm_model_unload(model)
