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
