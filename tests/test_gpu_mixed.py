"""configs[4] (DeepSeek-V2-Lite shape, Q8_0): the dense layer 0, then MoE layers with 64 routed
experts (softmax -> top-6, no renormalisation, x1.0) and the two always-on shared experts, as one
stack whose combine adds the shared FFN's output after the routed terms (umsx_stack_create_mixed).
All 27 layers bit for bit against the oracle at T = 1 and 5 (the per-stage kernels); the dense layer
and a MoE + shared layer at T = 2048 (the tensor-core prefill path) within the north-star tolerance
on sampled rows (tokens are independent of one another through a layer)."""
import importlib

import numpy as np
import pytest
import torch

from tests.helpers import C, bits, oracle_mixed_stack, to_cuda_bf16, umsx, x_bits

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 5e-3, 2e-2


def _mixed():
    import __graft_entry__ as ge
    pkg = ge.load_package()
    return importlib.import_module(pkg.__name__ + ".mixed")


def _close_all(stack, layers, shared):
    stack.close()
    for h in layers + [s for s in shared if s is not None]:
        h.close()


@pytest.mark.parametrize("tokens", [1, 5])
def test_deepseek_v2_lite_stack_bit_exact(oracle, tokens):
    mixed = _mixed()
    L = C.DEEPSEEK_V2_LITE.layers
    stack, layers, shared = mixed.deepseek_v2_lite_stack(L, max_tokens=8)
    xb = x_bits(oracle, C.DEEPSEEK_V2_LITE, tokens, stream=0xFFFF7)
    want = oracle_mixed_stack(oracle, xb, L)
    got = stack.forward(to_cuda_bf16(xb)).cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(want))
    # the stage-timed replay (a combine kernel of its own per layer) gives the same bits
    stack.set_timing(True)
    np.testing.assert_array_equal(bits(stack.forward(to_cuda_bf16(xb)).cpu().numpy()), bits(want))
    _close_all(stack, layers, shared)


@pytest.mark.parametrize("layer", [0, 1])
def test_deepseek_v2_lite_prefill_layer_t2048(oracle, layer):
    """One block layer at T = 2048 as a one-layer stack: layer 0 (the dense FFN) and layer 1 (64
    routed experts + the shared FFN fused into the combine), sampled rows within tolerance."""
    T = 2048
    if layer == 0:
        d = C.DEEPSEEK_V2_LITE_DENSE
        layers, shared = [umsx.MoeLayer(d.desc(T), synthetic=d.synthetic(layer=0))], [None]
    else:
        r, sh = C.DEEPSEEK_V2_LITE, C.DEEPSEEK_V2_LITE_SHARED
        layers = [umsx.MoeLayer(r.desc(T), synthetic=r.synthetic(layer=layer))]
        shared = [umsx.MoeLayer(sh.desc(T), synthetic=sh.synthetic(layer=layer))]
    stack = umsx.MoeStack(layers, max_tokens=T, shared=shared)
    xb = x_bits(oracle, C.DEEPSEEK_V2_LITE, T, stream=0xFFFF8)
    got = stack.forward(to_cuda_bf16(xb)).cpu().numpy()
    rows = np.unique(np.linspace(0, T - 1, 48).astype(np.int64))
    want = oracle_mixed_stack(oracle, xb[rows], 1, first=layer)
    err = got[rows].astype(np.float64) - want.astype(np.float64)
    rel = np.linalg.norm(err) / np.linalg.norm(want.astype(np.float64))
    scale = float(np.abs(want).max())
    assert rel <= REL_L2 and np.abs(err).max() <= MAX_ABS * max(1.0, scale), (rel, np.abs(err).max(), scale)
    _close_all(stack, layers, shared)
