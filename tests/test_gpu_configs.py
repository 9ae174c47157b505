"""The BASELINE configurations at their full shapes against the oracle (needs a B200).

configs[2] (GPT-OSS-120B-shaped: 128 MXFP4 experts, top-4, hidden = ffn = 2880, RMSNorm + residual)
through the one-launch decode kernels and the per-stage kernels, bit for bit; configs[1]
(Qwen3-30B-A3B-shaped Q8_0 layer) at its token counts T = 1 and 16 bit for bit, and T = 512 within
the north-star tolerance; configs[4]'s routed layer (DeepSeek-V2-Lite-shaped) at T = 2048 within
tolerance.  The oracle draws only the experts its routing selects (selected_host_weights), so the
full shapes stay cheap on the host; at many tokens it checks a sample of rows (tokens are
independent of one another in a MoE layer).
"""
import numpy as np
import pytest
import torch

from tests.helpers import (C, U, bf16_bits_to_f32, bits, oracle_desc, oracle_stack, selected_host_weights,
                           to_cuda_bf16, umsx, x_bits)

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 5e-3, 2e-2


def _close(got, want):
    err = got.astype(np.float64) - want.astype(np.float64)
    rel = np.linalg.norm(err) / max(np.linalg.norm(want.astype(np.float64)), 1e-30)
    return rel, float(np.abs(err).max())


@pytest.mark.parametrize("tokens", [1, 4])
def test_gpt_oss_120b_shape_stack_bit_exact(oracle, tokens):
    """Two configs[2] layers: the one-launch decode kernel (T = 1: one-token kernel, T = 4: the
    multi-token kernel) and the per-stage kernels (taken while stage timing is on) against the oracle."""
    cfg = C.GPT_OSS_120B
    L = 2
    xb = x_bits(oracle, cfg, tokens, stream=0xFFFF3)
    want = oracle_stack(oracle, cfg, xb, L)
    layers = [U.MoeLayer(cfg.desc(max_tokens=4), synthetic=cfg.synthetic(layer=l)) for l in range(L)]
    stack = umsx.MoeStack(layers, max_tokens=4)
    x = to_cuda_bf16(xb)
    launches = U.kernel_launches()
    fast = stack.forward(x).cpu().numpy()
    assert U.kernel_launches() - launches == 1, "expected the one-launch decode kernel"
    np.testing.assert_array_equal(bits(fast), bits(want))
    stack.set_timing(True)
    staged = stack.forward(x).cpu().numpy()
    np.testing.assert_array_equal(bits(staged), bits(want))
    stack.close()
    for l in layers:
        l.close()


@pytest.mark.parametrize("tokens", [1, 16])
def test_qwen3_30b_full_shape_bit_exact(oracle, tokens):
    """configs[1] (Q8_0, separate gate/up, SiLU, softmax -> top-8 -> renormalise) at T = 1 and 16."""
    cfg = C.QWEN3_30B
    xb = x_bits(oracle, cfg, tokens, stream=0xFFFF4)
    x32 = bf16_bits_to_f32(xb)
    desc = oracle_desc(cfg)
    ids, _, _ = oracle.route(desc, selected_host_weights(oracle, cfg, 0, []), x32)
    want = oracle.moe_layer(desc, selected_host_weights(oracle, cfg, 0, ids), x32, threads=16)
    layer = U.MoeLayer(cfg.desc(max_tokens=tokens), synthetic=cfg.synthetic())
    gi = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    gw = torch.empty((tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    out = layer.forward(to_cuda_bf16(xb), ids=gi, weights=gw).cpu().numpy()
    np.testing.assert_array_equal(gi.cpu().numpy(), want["ids"])
    np.testing.assert_array_equal(bits(gw.cpu().numpy()), bits(want["weights"]))
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    _, _, counts = layer.route(to_cuda_bf16(xb))
    np.testing.assert_array_equal(counts.cpu().numpy(), want["counts"])
    layer.close()


def _sampled_layer_check(oracle, cfg, tokens, sample, stream):
    """GPU layer at `tokens` rows; the oracle on `sample` of them (ids bit-exact, output within tolerance)."""
    xb = x_bits(oracle, cfg, tokens, stream=stream)
    layer = U.MoeLayer(cfg.desc(max_tokens=tokens), synthetic=cfg.synthetic())
    gi = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    out = layer.forward(to_cuda_bf16(xb), ids=gi).cpu().numpy()
    rows = np.unique(np.linspace(0, tokens - 1, sample).astype(np.int64))
    x32 = bf16_bits_to_f32(xb[rows])
    desc = oracle_desc(cfg)
    ids, _, _ = oracle.route(desc, selected_host_weights(oracle, cfg, 0, []), x32)
    want = oracle.moe_layer(desc, selected_host_weights(oracle, cfg, 0, ids), x32, threads=16)
    np.testing.assert_array_equal(gi.cpu().numpy()[rows], want["ids"])
    rel, mab = _close(out[rows], want["out"])
    scale = float(np.abs(want["out"]).max())
    layer.close()
    return rel, mab, scale


def test_qwen3_30b_full_shape_prefill_t512(oracle):
    """configs[1] at T = 512 (the tensor-core prefill path), every row checked."""
    rel, mab, scale = _sampled_layer_check(oracle, C.QWEN3_30B, 512, 512, 0xFFFF5)
    assert rel <= REL_L2 and mab <= MAX_ABS * max(1.0, scale), (rel, mab, scale)


def test_deepseek_v2_lite_routed_layer_t2048(oracle):
    """configs[4]'s routed layer (64 Q8_0 experts, top-6, softmax without renormalisation) at T = 2048,
    128 rows spread over the batch checked against the oracle."""
    rel, mab, scale = _sampled_layer_check(oracle, C.DEEPSEEK_V2_LITE, 2048, 128, 0xFFFF6)
    assert rel <= REL_L2 and mab <= MAX_ABS * max(1.0, scale), (rel, mab, scale)
