"""GGUF expert-slice loader (umsx_gguf_load_experts), on the CPU.

Follows the reference's load_gguf_experts contract (tools/engine/gguf_experts.cpp:45-140):
selected experts' packed slices and fp32 values from a (sharded) GGUF, biases as fp32,
and its validation errors.  Files are written with gguf-py, which also provides the
cross-check of the dequantized values (gguf.quants.dequantize).
"""
import os

import numpy as np
import pytest

from tests.helpers import U, bf16_bits_to_f32, host_weights, small_config, write_layer_gguf

gguf = pytest.importorskip("gguf")


def _cfg(quant, fused, bias):
    return small_config(hidden=128, intermediate=64, experts=6, top_k=2, quant=quant, fused_gate_up=fused,
                        has_bias=bias, has_router_bias=bias, seed=5)


def _qt(quant):
    return gguf.GGMLQuantizationType.MXFP4 if quant == U.QUANT_MXFP4 else gguf.GGMLQuantizationType.Q8_0


@pytest.mark.parametrize("quant", [U.QUANT_MXFP4, U.QUANT_Q8_0])
def test_selected_slices_match_gguf_py(oracle, tmp_path, quant):
    cfg = _cfg(quant, fused=quant == U.QUANT_MXFP4, bias=True)
    w = host_weights(oracle, cfg, layer=3)
    path = str(tmp_path / "layer.gguf")
    write_layer_gguf([path], 3, w, quant, cfg.hidden, cfg.intermediate)
    ids = [4, 1, 5]
    got = U.load_gguf_experts(path, 3, ids)
    I = cfg.intermediate
    gate = w.gate if w.gate_up is None else w.gate_up[:, :I]
    up = w.up if w.gate_up is None else w.gate_up[:, I:]
    src = {"gate": gate, "up": up, "down": w.down}
    gb = bf16_bits_to_f32(w.gate_up_bias)
    bias = {"gate": gb[:, :I], "up": gb[:, I:], "down": bf16_bits_to_f32(w.down_bias)}
    assert (got["hidden"], got["intermediate"], got["experts"]) == (cfg.hidden, I, cfg.experts)
    for name in ("gate", "up", "down"):
        d = got[name]
        assert d["type"] == quant
        want = np.ascontiguousarray(src[name][ids]).reshape(len(ids), -1)
        np.testing.assert_array_equal(d["packed"], want)
        ref = gguf.quants.dequantize(np.ascontiguousarray(src[name][ids]), _qt(quant))
        np.testing.assert_array_equal(d["values"].view(np.uint32), ref.astype(np.float32).view(np.uint32))
        np.testing.assert_array_equal(d["bias"], bias[name][ids])


def test_sharded_q8_0_f16_bias_and_no_values(oracle, tmp_path):
    cfg = _cfg(U.QUANT_Q8_0, fused=False, bias=True)
    w = host_weights(oracle, cfg, layer=0)
    paths = [str(tmp_path / "m-00001-of-00002.gguf"), str(tmp_path / "m-00002-of-00002.gguf")]
    write_layer_gguf(paths, 0, w, U.QUANT_Q8_0, cfg.hidden, cfg.intermediate, split_at=3, bias_dtype=np.float16)
    got = U.load_gguf_experts(paths[0], 0, [0, 5], dequantize=False)
    np.testing.assert_array_equal(got["down"]["packed"], w.down[[0, 5]].reshape(2, -1))
    assert "values" not in got["gate"]
    gb = bf16_bits_to_f32(w.gate_up_bias)[[0, 5]]
    np.testing.assert_array_equal(got["up"]["bias"], gb[:, cfg.intermediate:].astype(np.float16).astype(np.float32))
    # without the second shard the experts' tensors are missing
    os.rename(paths[1], paths[1] + ".moved")
    with pytest.raises(U.UmsxError, match="missing or not readable"):
        U.load_gguf_experts(paths[0], 0, [0])


def test_validation_errors(oracle, tmp_path):
    cfg = _cfg(U.QUANT_MXFP4, fused=False, bias=False)
    w = host_weights(oracle, cfg, layer=1)
    path = str(tmp_path / "layer.gguf")
    write_layer_gguf([path], 1, w, U.QUANT_MXFP4, cfg.hidden, cfg.intermediate, extra_kv=False)
    for ids, msg in (([], "invalid layer"), (list(range(17)), "invalid layer"), ([1, 1], "invalid layer"),
                     ([6], "outside tensor")):
        with pytest.raises(U.UmsxError, match=msg):
            U.load_gguf_experts(path, 1, ids)
    with pytest.raises(U.UmsxError, match="invalid layer"):
        U.load_gguf_experts(path, 4096, [0])
    with pytest.raises(U.UmsxError, match="missing"):
        U.load_gguf_experts(path, 2, [0])  # no such layer
    got = U.load_gguf_experts(path, 1, [2])
    assert "bias" not in got["gate"]
    raw = open(path, "rb").read()
    bad = str(tmp_path / "bad.gguf")
    open(bad, "wb").write(b"GGUX" + raw[4:])
    with pytest.raises(U.UmsxError, match="not a GGUF file"):
        U.load_gguf_experts(bad, 1, [0])
    open(bad, "wb").write(raw[: len(raw) - 100])
    with pytest.raises(U.UmsxError, match="exceeds shard"):
        U.load_gguf_experts(bad, 1, [0])
    open(bad, "wb").write(raw[:40])
    with pytest.raises(U.UmsxError, match="could not be read"):
        U.load_gguf_experts(bad, 1, [0])
    # extents that each pass the per-dimension bound but whose product overflows int64
    name = b"blk.1.ffn_gate_exps.weight"
    at = raw.index(name) + len(name)
    n_dims = int.from_bytes(raw[at:at + 4], "little")
    assert n_dims == 3
    huge = (1 << 40).to_bytes(8, "little")
    patched = raw[:at + 4] + huge + huge + raw[at + 20:]
    open(bad, "wb").write(patched)
    with pytest.raises(U.UmsxError, match="element count overflows"):
        U.load_gguf_experts(bad, 1, [0])


def test_create_rejects_a_descriptor_that_does_not_match(oracle, tmp_path):
    cfg = _cfg(U.QUANT_MXFP4, fused=True, bias=True)
    w = host_weights(oracle, cfg, layer=0)
    path = str(tmp_path / "layer.gguf")
    write_layer_gguf([path], 0, w, U.QUANT_MXFP4, cfg.hidden, cfg.intermediate)
    import dataclasses
    for over, msg in (({"experts": 8}, "router shape"), ({"quant": U.QUANT_Q8_0}, "quantization"),
                      ({"has_bias": False}, "has_bias"), ({"has_router_bias": False}, "router bias")):
        bad = dataclasses.replace(cfg, **over)
        with pytest.raises(U.UmsxError, match=msg):
            U.MoeLayer(bad.desc(4), gguf=(path, 0))
