"""GGUF container reader (cybel_b200/gguf_file.py) against files written by
gguf-py's GGUFWriter and read back by gguf-py's GGUFReader (the library the
reference loads its models with, core/model/gguf_loader.py:27,178).

* metadata of every value type, tensor dims, types and bytes: identical to
  what was written and to GGUFReader's view;
* quantized tensors come back as the rows the kernels consume (bytes equal);
* a llama-architecture file maps onto the decode stack's weights exactly;
* malformed files and unsupported layouts raise GGUFError.
"""

from __future__ import annotations

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")


def _write(path, arch, kv, tensors):
    w = gguf.GGUFWriter(str(path), arch)
    for key, (kind, val) in kv.items():
        getattr(w, f"add_{kind}")(key, val)
    for name, (arr, qt) in tensors.items():
        if qt is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType(qt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _packed(qt, n, k, seed):
    from cybel_b200 import quantize as Q

    return Q.quantize(np.random.default_rng(seed).normal(0.0, 0.02, size=(n, k)).astype(np.float32), qt)


def test_reader_matches_writer_and_gguf_py(tmp_path):
    from cybel_b200.gguf_file import GGUFFile

    tensors = {
        "a.q4k": (_packed(12, 48, 512, 0), 12),
        "a.q6k": (_packed(14, 7, 256, 1), 14),
        "a.q80": (_packed(8, 9, 96, 2), 8),
        "a.q40": (_packed(2, 5, 64, 3), 2),
        "a.f32": (np.random.default_rng(4).standard_normal(33).astype(np.float32), None),
        "a.f16": (np.random.default_rng(5).standard_normal((3, 40)).astype(np.float16), None),
    }
    kv = {"t.u32": ("uint32", 7), "t.f32": ("float32", 0.25), "t.str": ("string", "héllo"),
          "t.bool": ("bool", True), "t.i64": ("int64", -5), "t.ints": ("array", [1, 2, 3]),
          "t.strs": ("array", ["x", "yz"])}
    path = tmp_path / "m.gguf"
    _write(path, "llama", kv, tensors)

    f = GGUFFile(path)
    assert f.metadata["general.architecture"] == "llama"
    assert f.metadata["t.u32"] == 7 and f.metadata["t.str"] == "héllo" and f.metadata["t.bool"] is True
    assert f.metadata["t.f32"] == pytest.approx(0.25) and f.metadata["t.i64"] == -5
    assert f.metadata["t.ints"] == [1, 2, 3] and f.metadata["t.strs"] == ["x", "yz"]
    for name, (arr, qt) in tensors.items():
        t = f.tensors[name]
        if qt is not None:
            assert t.ggml_type == qt and t.dims == (arr.shape[1] * {12: 256, 14: 256, 8: 32, 2: 32}[qt] //
                                                    {12: 144, 14: 210, 8: 34, 2: 18}[qt], arr.shape[0])
            assert np.array_equal(f.raw(name), arr)
            qm = f.quantized(name)
            assert qm.qtype == qt and qm.shape == t.dims and np.array_equal(qm.data, arr)
        else:
            assert np.array_equal(f.array(name), arr.astype(np.float32))
    # gguf-py's own view of the same file
    r = gguf.GGUFReader(str(path))
    for t in r.tensors:
        mine = f.tensors[t.name]
        assert mine.ggml_type == int(t.tensor_type.value)
        assert mine.dims == tuple(int(d) for d in t.shape)
        assert mine.offset == int(t.data_offset)
        assert np.array_equal(f.raw(t.name).reshape(-1), np.asarray(t.data).view(np.uint8).reshape(-1))


def _tiny_llama(tmp_path, linear_qt=12, mixed=False, tied=False, name="llama.gguf"):
    from cybel_b200.decode import StackShape, random_layer, random_rows

    shape = StackShape(layers=2, hidden=512, heads=4, kv_heads=2, ffn=768, vocab=320, rope_theta=10000.0,
                       linear_qtype=linear_qt, head_qtype=14, embed_qtype=14)
    rng = np.random.default_rng(11)
    layers = [random_layer(shape, rng) for _ in range(shape.layers)]
    if mixed:
        layers[1]["wv"] = random_rows(14, shape.kv_dim, shape.hidden, rng)
    embed = random_rows(14, shape.vocab, shape.hidden, rng, std=1.0)
    head = random_rows(14, shape.vocab, shape.hidden, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    names = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "w_gate": "ffn_gate",
             "w_up": "ffn_up", "w_down": "ffn_down"}
    tensors = {"token_embd.weight": (embed, 14), "output_norm.weight": (out_norm, None)}
    if not tied:
        tensors["output.weight"] = (head, 14)
    for i, lay in enumerate(layers):
        for key, n in names.items():
            qt = 14 if (mixed and i == 1 and key == "wv") else linear_qt
            tensors[f"blk.{i}.{n}.weight"] = (lay[key], qt)
        tensors[f"blk.{i}.attn_norm.weight"] = (lay["attn_norm"], None)
        tensors[f"blk.{i}.ffn_norm.weight"] = (lay["ffn_norm"], None)
    kv = {"llama.block_count": ("uint32", 2), "llama.embedding_length": ("uint32", 512),
          "llama.attention.head_count": ("uint32", 4), "llama.attention.head_count_kv": ("uint32", 2),
          "llama.feed_forward_length": ("uint32", 768), "llama.rope.freq_base": ("float32", 10000.0),
          "llama.attention.layer_norm_rms_epsilon": ("float32", 1e-5)}
    path = tmp_path / name
    _write(path, "llama", kv, tensors)
    return path, shape, layers, embed, (embed if tied else head), out_norm


@pytest.mark.parametrize("tied", [False, True])
def test_llama_file_maps_onto_decode_stack(tmp_path, tied):
    from cybel_b200.gguf_file import load_llama_stack

    path, shape, layers, embed, head, out_norm = _tiny_llama(tmp_path, tied=tied)
    s2, l2, e2, h2, n2 = load_llama_stack(path)
    assert (s2.layers, s2.hidden, s2.heads, s2.kv_heads, s2.ffn, s2.vocab) == (2, 512, 4, 2, 768, 320)
    assert (s2.linear_qtype, s2.head_qtype, s2.embedding_qtype) == (12, 14, 14)
    assert s2.rope_theta == pytest.approx(10000.0) and s2.eps == pytest.approx(1e-5)
    assert np.array_equal(e2, embed) and np.array_equal(h2, head) and np.array_equal(n2, out_norm)
    for a, b in zip(layers, l2):
        assert set(a) == set(b)
        for key in a:
            assert np.array_equal(a[key], b[key]), key


def test_malformed_and_unsupported_files(tmp_path):
    from cybel_b200.gguf_file import GGUFError, GGUFFile, load_llama_stack

    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(64))
    with pytest.raises(GGUFError):
        GGUFFile(bad)
    path, *_ = _tiny_llama(tmp_path)
    blob = path.read_bytes()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(blob[: len(blob) // 2])
    with pytest.raises(GGUFError):
        GGUFFile(cut)
    f = GGUFFile(path)
    with pytest.raises(GGUFError):
        f.quantized("blk.0.attn_norm.weight")  # a float tensor
    with pytest.raises(GGUFError):
        f.array("blk.0.attn_q.weight")  # a quantized tensor
    mixed, *_ = _tiny_llama(tmp_path, mixed=True, name="mixed.gguf")
    with pytest.raises(GGUFError):
        load_llama_stack(mixed)


@pytest.mark.gpu
def test_decode_stack_from_gguf_equals_arrays(tmp_path):
    """The same weights through the file and from arrays: the same logits
    (same kernels on the same bytes; 1e-6 relative allows for a reduction
    order that depends on CTA arrival)."""
    from cybel_b200.decode import DecodeStack

    path, shape, layers, embed, head, out_norm = _tiny_llama(tmp_path)
    a = DecodeStack.from_gguf(path, 32)
    b = DecodeStack(shape, 32, layers, embed, head, out_norm)
    for pos, tok in enumerate([3, 17, 300, 0, 42]):
        a.set_token(tok)
        b.set_token(tok)
        a.step(pos)
        b.step(pos)
        la, lb = a.logits.cpu().numpy(), b.logits.cpu().numpy()
        assert np.max(np.abs(la - lb)) <= 1e-6 * np.max(np.abs(lb)), pos
