# SPDX-License-Identifier: MIT
"""GGUF files (include/qh_gguf.h): a synthetic blob written with
qh_gguf_write reads back identically through qh_gguf_load, and the
reference's own loader (gguf_open slm/gguf.c:172, slm_load_config
slm/qwen.c:59, slm_load_weights slm/qwen.c:174) reads the same file into
the same config and steps the same logits, bit for bit, as the reference
built over the in-memory blob. Malformed files are rejected with a status,
as gguf_open rejects them (slm/gguf.c:180-260).
"""
import ctypes as C
import os

import numpy as np
import pytest

CFG_FIELDS = ["n_layers", "hidden", "ffn", "vocab", "n_heads", "n_kv_heads", "head_dim",
              "rope_dim", "rope_theta", "norm_eps", "gdn_heads", "gdn_head_dim", "conv_kernel",
              "full_attn_interval", "max_pos"]


def cfg_tuple(c):
    return tuple(getattr(c, f) for f in CFG_FIELDS) + tuple(c.rope_sections)


def tensor_bytes(blob):
    return [(n, t, s, C.string_at(p, nb)) for n, t, s, p, nb in blob.tensors()]


@pytest.fixture(scope="module")
def written(qh, tmp_path_factory):
    cfg = qh.host.slm_config(64, n_layers=4, vocab=1024)
    blob = qh.host.Blob(cfg, 0x6611F)
    path = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    blob.write_gguf(path)
    return cfg, blob, path


def test_roundtrip_config_and_tensors(qh, written):
    cfg, blob, path = written
    back = qh.host.Blob.from_gguf(path)
    assert cfg_tuple(back.cfg) == cfg_tuple(cfg)
    a, b = tensor_bytes(blob), tensor_bytes(back)
    assert [x[:3] for x in a] == [x[:3] for x in b]
    for (name, _, _, da), (_, _, _, db) in zip(a, b):
        assert da == db, name
    back.close()


def test_data_alignment(written):
    """Tensor data starts on 32-byte boundaries (general.alignment)."""
    _, blob, path = written
    size = os.path.getsize(path)
    total = sum((nb + 31) // 32 * 32 for *_, nb in blob.tensors())
    assert size >= total and (size - total) % 32 == 0


def test_max_pos_cap(qh, written):
    cfg, _, path = written
    back = qh.host.Blob.from_gguf(path, max_pos_cap=16)
    assert back.cfg.max_pos == 16
    back.close()
    back = qh.host.Blob.from_gguf(path, max_pos_cap=100000)
    assert back.cfg.max_pos == cfg.max_pos  # context_length wins when smaller
    back.close()


def _status(qh, path):
    cfg, h = qh.SlmConfig(), C.c_void_p()
    st = qh.lib().qh_gguf_load(path.encode(), 0, C.byref(cfg), C.byref(h))
    if h.value:
        qh.lib().qh_blob_free(h)
    return st


def test_malformed_rejected(qh, written, tmp_path):
    _, _, path = written
    raw = open(path, "rb").read()
    cases = {
        "magic": b"XGUF" + raw[4:],
        "version": raw[:4] + (1).to_bytes(4, "little") + raw[8:],
        "truncated_header": raw[:40],
        "truncated_data": raw[:len(raw) - 100],
        "empty": b"",
    }
    for name, data in cases.items():
        p = str(tmp_path / f"{name}.gguf")
        open(p, "wb").write(data)
        assert _status(qh, p) == -1, name
    assert _status(qh, str(tmp_path / "missing.gguf")) == -1


def test_other_architecture_unsupported(qh, written, tmp_path):
    _, _, path = written
    raw = open(path, "rb").read()
    i = raw.index(b"qwen35")
    p = str(tmp_path / "llama.gguf")
    open(p, "wb").write(raw[:i] + b"llama3" + raw[i + 6:])
    assert _status(qh, p) == -2


def test_reference_loader_reads_it(ref, written):
    """The reference's loader sees the config written and steps the same
    logits as the reference over the in-memory tensors."""
    from oracle.oracle import RefModel
    cfg, blob, path = written
    rg, ic, fc = RefModel.from_gguf(ref, path)
    want = [cfg.n_layers, cfg.hidden, cfg.ffn, cfg.vocab, cfg.n_heads, cfg.n_kv_heads,
            cfg.head_dim, cfg.rope_dim, *list(cfg.rope_sections), cfg.gdn_heads,
            cfg.gdn_head_dim, cfg.conv_kernel, cfg.full_attn_interval, cfg.max_pos]
    assert list(ic) == want
    assert fc[0] == np.float32(cfg.rope_theta) and fc[1] == np.float32(cfg.norm_eps)
    rm = RefModel(ref, cfg, blob.tensors())
    tok = 7
    for pos in range(12):
        a0, l0 = rm.step(tok, pos, want_logits=True)
        a1, l1 = rg.step(tok, pos, want_logits=True)
        assert a0 == a1 and np.array_equal(l0, l1), pos
        tok = a0
    rm.close()
    rg.close()


@pytest.mark.gpu
def test_device_model_from_gguf(qh, cuda, written):
    """Greedy picks of the device model over the loaded blob equal those over
    the blob that was written."""
    cfg, blob, path = written
    back = qh.host.Blob.from_gguf(path)
    prompt = np.array([[3, 1, 4, 1, 5, 9, 2, 6]], np.int32)
    outs = []
    for b in (blob, back):
        slm = qh.host.Slm(b.cfg, b, 1)
        outs.append(slm.generate(prompt, 24).copy())
        slm.close()
    back.close()
    assert np.array_equal(outs[0], outs[1])


@pytest.fixture(scope="module", params=[1, 2], ids=["q4_k_m_mix", "all_types"])
def written_mix(qh, tmp_path_factory, request):
    """A GGUF whose weights carry the released Q4_K_M file's types (Q5_K,
    Q6_K, Q8_0 beside Q4_K), or every type the matmuls compute (F32 too)."""
    cfg = qh.host.slm_config(48, n_layers=4, vocab=1024)
    blob = qh.host.Blob(cfg, 0x6612F + request.param, mix=request.param)
    path = str(tmp_path_factory.mktemp("gguf") / f"mix{request.param}.gguf")
    blob.write_gguf(path)
    return cfg, blob, path, request.param


def test_mix_types_written_and_read_back(qh, written_mix):
    cfg, blob, path, mix = written_mix
    types = {n: t for n, t, *_ in blob.tensors()}
    if mix == 1:
        assert types["blk.0.attn_qkv.weight"] == 13 and types["blk.0.ssm_alpha.weight"] == 8
        assert types["blk.3.attn_v.weight"] == 14 and types["blk.3.attn_q.weight"] == 13
    else:
        assert types["token_embd.weight"] == 0 and types["blk.3.attn_k.weight"] == 0
    back = qh.host.Blob.from_gguf(path)
    assert [x[:3] for x in tensor_bytes(back)] == [x[:3] for x in tensor_bytes(blob)]
    back.close()


def test_reference_loader_reads_mix(ref, written_mix):
    """The reference's loader binds the mixed-type file; its steps equal the
    reference over the in-memory tensors (matmul_dispatch per type)."""
    from oracle.oracle import RefModel
    cfg, blob, path, _ = written_mix
    rg, _, _ = RefModel.from_gguf(ref, path)
    rm = RefModel(ref, cfg, blob.tensors())
    tok = 11
    for pos in range(8):
        a0, l0 = rm.step(tok, pos, want_logits=True)
        a1, l1 = rg.step(tok, pos, want_logits=True)
        assert a0 == a1 and np.array_equal(l0, l1), pos
        tok = a0
    rm.close()
    rg.close()


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 3, 12])
def test_device_model_mix_matches_reference_gguf(qh, cuda, ref, written_mix, B):
    """The device model over the loaded mixed-type file (every projection by
    its own GGUF type; B = 12 runs the K-quants on the tensor-core GEMM) gives
    the logits, bit for bit, of the stock reference loading the same file."""
    from oracle.oracle import RefModel
    cfg, _, path, _ = written_mix
    back = qh.host.Blob.from_gguf(path)
    rng = np.random.default_rng(B)
    n_prompt, n_new = 6, 10
    prompts = rng.integers(0, cfg.vocab, (B, n_prompt)).astype(np.int32)
    slm = qh.host.Slm(back.cfg, back, B)
    gl = []
    tok = prompts[:, 0].copy()
    preds = []
    for pos in range(n_prompt + n_new - 1):
        nxt, lg = slm.step(tok, pos, want_logits=True)
        preds.append(nxt.copy())
        gl.append(lg.copy())
        tok = prompts[:, pos + 1] if pos + 1 < n_prompt else nxt
    slm.close()
    preds = np.stack(preds, 1)
    for b in sorted({0, B - 1}):
        rg, _, _ = RefModel.from_gguf(ref, path)
        t = prompts[b, 0]
        for pos in range(n_prompt + n_new - 1):
            a, lr = rg.step(int(t), pos, want_logits=True)
            assert a == preds[b, pos], f"seq {b} step {pos}: pick {preds[b, pos]} vs reference {a}"
            assert np.array_equal(gl[pos][b].view(np.uint32), lr.view(np.uint32)), f"seq {b} step {pos} logits"
            t = prompts[b, pos + 1] if pos + 1 < n_prompt else a
        rg.close()
    back.close()


@pytest.mark.gpu
def test_model_rejects_a_type_it_does_not_compute(qh, cuda):
    """Tensors are checked when the model is created: an embedding table of
    a type the row reader does not take (Q4_K; the reference reads only Q6_K
    or F32 rows there, slm/qwen.c:885-907) is QH_ERR_UNSUPPORTED, a matrix of
    another shape QH_ERR_INVALID; a tensor of a type no matmul computes (F16)
    is refused when added (the reference aborts on it, slm/model.c:259-261)."""
    cfg = qh.host.slm_config(16, n_layers=4, vocab=512)
    src = qh.host.Blob(cfg, 5)
    for bad in ("embd_type", "shape"):
        b = qh.host.Blob.empty(cfg)
        for name, typ, shape, ptr, nb in src.tensors():
            data = C.string_at(ptr, nb)
            if bad == "embd_type" and name == "token_embd.weight":
                typ = 12
                data = bytes((shape[0] // 256) * 144 * shape[1])
            if bad == "shape" and name == "blk.0.ffn_gate.weight":
                shape = (shape[0], shape[1] - 256)
                data = data[:nb // cfg.ffn * (cfg.ffn - 256)]
            b.add(name, typ, shape, data)
        with pytest.raises(qh.QHError) as e:
            qh.host.Slm(cfg, b, 1)
        assert e.value.status == (-2 if bad == "embd_type" else -1), bad
        b.close()
    b = qh.host.Blob.empty(cfg)
    with pytest.raises(qh.QHError) as e:
        b.add("x", 1, (256, 4), bytes(256 * 4 * 2))
    assert e.value.status == -2
    b.close()
    src.close()
