"""configs[4] (DeepSeek-V2-Lite shape, Q8_0): a MoE layer with the always-on shared experts and
the dense FFN of layer 0, through one-expert top-1 layers, bit for bit against the oracle (routed
layer + shared FFN added in fp32; the dense FFN as the oracle's one-expert layer)."""
import importlib

import numpy as np
import pytest
import torch

from tests.helpers import C, bf16_bits_to_f32, bits, host_weights, oracle_desc, to_cuda_bf16, umsx, x_bits

pytestmark = pytest.mark.gpu


def _mixed():
    import __graft_entry__ as ge
    pkg = ge.load_package()
    return importlib.import_module(pkg.__name__ + ".mixed")


@pytest.mark.parametrize("tokens", [1, 5])
def test_shared_expert_block_bit_exact(oracle, tokens):
    mixed = _mixed()
    rc, sc = C.DEEPSEEK_V2_LITE, C.DEEPSEEK_V2_LITE_SHARED
    xb = x_bits(oracle, rc, tokens)
    x = bf16_bits_to_f32(xb)
    want_r = oracle.moe_layer(oracle_desc(rc), host_weights(oracle, rc, layer=1), x, threads=8)
    want_s = oracle.moe_layer(oracle_desc(sc), host_weights(oracle, sc, layer=1), x, threads=8)
    assert (want_s["ids"] == 0).all() and (want_s["weights"] == 1.0).all()
    want = (want_r["out"] + want_s["out"]).astype(np.float32)
    routed = umsx.MoeLayer(rc.desc(8), synthetic=rc.synthetic(layer=1))
    shared = umsx.MoeLayer(sc.desc(8), synthetic=sc.synthetic(layer=1))
    got = mixed.SharedExpertBlock(routed, shared).forward(to_cuda_bf16(xb)).cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(want))
    routed.close()
    shared.close()


def test_dense_layer0_ffn_bit_exact(oracle):
    mixed = _mixed()
    dc = C.DEEPSEEK_V2_LITE_DENSE
    tokens = 3
    xb = x_bits(oracle, dc, tokens)
    want = oracle.moe_layer(oracle_desc(dc), host_weights(oracle, dc, layer=0), bf16_bits_to_f32(xb), threads=8)
    layer = umsx.MoeLayer(dc.desc(4), synthetic=dc.synthetic(layer=0))
    got = mixed.DenseFFN(layer).forward(to_cuda_bf16(xb)).cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(want["out"]))
    layer.close()
