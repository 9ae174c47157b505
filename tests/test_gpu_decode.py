"""Persistent decode kernel (one cooperative launch per forward, T <= 4) against the
oracle and against the per-stage kernels on the same inputs."""
import numpy as np
import pytest
import torch

from tests.helpers import (U, bf16_bits_to_f32, bits, host_weights, oracle_desc, small_config, to_cuda_bf16,
                           umsx, x_bits)

pytestmark = pytest.mark.gpu


def _oracle_stack(oracle, cfg, xb, n_layers):
    h = bf16_bits_to_f32(xb).copy()
    for l in range(n_layers):
        xn = oracle.rmsnorm(h, 1e-5)
        h = (h + oracle.moe_layer(oracle_desc(cfg), host_weights(oracle, cfg, layer=l), xn, threads=8)["out"])
        h = h.astype(np.float32)
    return h


@pytest.mark.parametrize("tokens", [1, 2, 4])
def test_decode_layer_bit_exact(oracle, tokens):
    cfg = small_config()
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, tokens)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=8)
    layer = U.MoeLayer(cfg.desc(8), synthetic=cfg.synthetic())
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    wt = torch.empty((tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    launches = U.kernel_launches()
    out = layer.forward(to_cuda_bf16(xb), ids=ids, weights=wt).cpu().numpy()
    assert U.kernel_launches() - launches == 1, "expected the single persistent launch"
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    np.testing.assert_array_equal(bits(wt.cpu().numpy()), bits(want["weights"]))
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    layer.close()


def test_decode_low_block_exponents_bit_exact(oracle):
    """Blocks with exponent bytes 0, 1 and 2 (subnormal block scales for 0 and 1): such a layer takes
    the general scale rule instead of the normal-scale form, and the one-launch kernel stays bit-exact."""
    from tests.helpers import weights_dict
    cfg = small_config()
    import dataclasses
    w = host_weights(oracle, cfg)
    w = dataclasses.replace(w, gate_up=w.gate_up.copy(), down=w.down.copy())
    rng = np.random.default_rng(5)
    for arr in (w.gate_up, w.down):
        blocks = arr.reshape(-1, 17)
        idx = rng.choice(blocks.shape[0], size=blocks.shape[0] // 8, replace=False)
        blocks[idx, 0] = rng.integers(0, 3, size=idx.size, dtype=np.uint8)
    xb = x_bits(oracle, cfg, 1)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=8)
    layer = U.MoeLayer(cfg.desc(1), weights_dict(w))
    launches = U.kernel_launches()
    out = layer.forward(to_cuda_bf16(xb)).cpu().numpy()
    assert U.kernel_launches() - launches == 1, "expected the single persistent launch"
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    layer.close()


@pytest.mark.parametrize("tokens", [1, 3])
def test_decode_stack_bit_exact(oracle, tokens):
    cfg = small_config()
    L = 3
    layers = [U.MoeLayer(cfg.desc(1), synthetic=cfg.synthetic(layer=l)) for l in range(L)]
    stack = umsx.MoeStack(layers, max_tokens=8)
    xb = x_bits(oracle, cfg, tokens)
    want = _oracle_stack(oracle, cfg, xb, L)
    launches = U.kernel_launches()
    got = stack.forward(to_cuda_bf16(xb)).cpu().numpy()
    assert U.kernel_launches() - launches == 1
    np.testing.assert_array_equal(bits(got), bits(want))
    hostout = torch.empty((tokens, cfg.hidden), dtype=torch.float32).pin_memory()
    stack.forward_host(torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).pin_memory(), hostout)
    np.testing.assert_array_equal(bits(hostout.numpy()), bits(want))
    stack.close()
    for l in layers:
        l.close()


def test_decode_matches_per_stage_path_gpt_oss_120b_shape():
    """Two GPT-OSS-120B-shaped layers (128 experts, top-4, 2880): the persistent kernel
    and the per-stage kernels (taken while stage timing is on) give identical bits."""
    from tests.helpers import C
    cfg = C.GPT_OSS_120B
    layers = [U.MoeLayer(cfg.desc(max_tokens=1), synthetic=cfg.synthetic(layer=l)) for l in range(2)]
    stack = umsx.MoeStack(layers, max_tokens=4)
    rng = np.random.default_rng(7)
    for tokens in (1, 4):
        x = torch.from_numpy(rng.standard_normal((tokens, cfg.hidden)).astype(np.float32)).to(torch.bfloat16).cuda()
        stack.set_timing(False)
        fast = stack.forward(x).cpu().numpy()
        stack.set_timing(True)
        staged = stack.forward(x).cpu().numpy()
        np.testing.assert_array_equal(bits(fast), bits(staged))
    stack.close()
    for l in layers:
        l.close()


@pytest.mark.parametrize("tokens", [1, 5])
def test_nan_input_routes_to_valid_experts(oracle, tokens):
    """A NaN in x makes every logit of that token NaN; NaN ranks lowest, so the token
    goes to experts 0..k-1 (as in the oracle) instead of to an invalid index.  T=1 takes
    the persistent kernel, T=5 the per-stage kernels."""
    cfg = small_config()
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, tokens).copy()
    xb[0, 3] = 0x7FC0  # bf16 quiet NaN
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=8)
    layer = U.MoeLayer(cfg.desc(8), synthetic=cfg.synthetic())
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    wt = torch.empty((tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    layer.forward(to_cuda_bf16(xb), ids=ids, weights=wt)
    torch.cuda.synchronize()
    got = ids.cpu().numpy()
    np.testing.assert_array_equal(got, want["ids"])
    np.testing.assert_array_equal(got[0], np.arange(cfg.top_k))
    layer.close()


# ---- one token: the one-token kernel (k_decode1) at assorted shapes --------------------------

_T1_SHAPES = [dict(), dict(hidden=320, intermediate=128, experts=16, top_k=8), dict(hidden=192, intermediate=320, experts=200, top_k=3)]


@pytest.mark.parametrize("shape", range(len(_T1_SHAPES)))
def test_one_token_layer_bit_exact(oracle, shape):
    """The shapes cover a partial last ring stage (5 block pairs), top-8, and more experts than
    CTAs (two router rows on some CTAs)."""
    cfg = small_config(**_T1_SHAPES[shape])
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, 1)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=8)
    layer = U.MoeLayer(cfg.desc(4), synthetic=cfg.synthetic())
    ids = torch.empty((1, cfg.top_k), dtype=torch.int32, device="cuda")
    wt = torch.empty((1, cfg.top_k), dtype=torch.float32, device="cuda")
    launches = U.kernel_launches()
    out = layer.forward(to_cuda_bf16(xb), ids=ids, weights=wt).cpu().numpy()
    assert U.kernel_launches() - launches == 1
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    np.testing.assert_array_equal(bits(wt.cpu().numpy()), bits(want["weights"]))
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    layer.close()


def test_one_token_stack_bit_exact(oracle):
    cfg = small_config()
    L = 4
    layers = [U.MoeLayer(cfg.desc(1), synthetic=cfg.synthetic(layer=l)) for l in range(L)]
    stack = umsx.MoeStack(layers, max_tokens=1)
    xb = x_bits(oracle, cfg, 1)
    want = _oracle_stack(oracle, cfg, xb, L)
    got = stack.forward(to_cuda_bf16(xb)).cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(want))
    stack.close()
    for l in layers:
        l.close()


def test_one_token_full_size_gpt_oss_20b_layer(oracle):
    """configs[0] shapes (2880 / 2880, 32 experts, top-4) through the one-token kernel."""
    from tests.helpers import C
    cfg = C.GPT_OSS_20B
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, 1)
    want = oracle.moe_layer(oracle_desc(cfg), w, bf16_bits_to_f32(xb), threads=16)
    layer = U.MoeLayer(cfg.desc(1), synthetic=cfg.synthetic())
    out = layer.forward(to_cuda_bf16(xb)).cpu().numpy()
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    layer.close()
