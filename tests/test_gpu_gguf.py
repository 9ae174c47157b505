"""Layers created from GGUF checkpoints (umsx_moe_create_gguf) on the GPU, through the C ABI.

A layer read from a GGUF file must compute exactly what the same weights passed to
umsx_moe_create compute: the file's fp32 biases are chosen bf16-representable so both
creation paths hold identical values, and every output must match bit for bit (the
weights-array path is itself bit-exact with the oracle in test_gpu_parity.py).
"""
import numpy as np
import pytest

from tests.helpers import U, bits, host_weights, small_config, to_cuda_bf16, weights_dict, write_layer_gguf, x_bits

torch = pytest.importorskip("torch")
pytest.importorskip("gguf")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("quant,fused,bias,shards", [(U.QUANT_MXFP4, True, True, 1), (U.QUANT_MXFP4, False, True, 2),
                                                      (U.QUANT_Q8_0, False, False, 2)])
def test_gguf_layer_matches_array_layer(oracle, tmp_path, quant, fused, bias, shards):
    cfg = small_config(hidden=256, intermediate=192, experts=8, top_k=2, quant=quant, fused_gate_up=fused,
                       has_bias=bias, has_router_bias=bias, seed=21,
                       **({} if quant == U.QUANT_MXFP4 else dict(routing=U.ROUTE_SOFTMAX_TOPK_NORM,
                                                                   activation=U.ACT_SILU)))
    w = host_weights(oracle, cfg, layer=2)
    paths = [str(tmp_path / "l.gguf")] if shards == 1 else \
        [str(tmp_path / "l-00001-of-00002.gguf"), str(tmp_path / "l-00002-of-00002.gguf")]
    write_layer_gguf(paths, 2, w, quant, cfg.hidden, cfg.intermediate, split_at=2)
    a = U.MoeLayer(cfg.desc(64), weights_dict(w))
    g = U.MoeLayer(cfg.desc(64), gguf=(paths[0], 2))
    try:
        for T in (1, 5, 64):
            x = to_cuda_bf16(x_bits(oracle, cfg, T, stream=0xABC0 + T))
            ya, yg = a.forward(x), g.forward(x)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(bits(yg.cpu().numpy()), bits(ya.cpu().numpy()), err_msg=f"T={T}")
    finally:
        a.close()
        g.close()
