"""configs[3] load skew (needs a B200): Qwen3-30B-A3B layer shapes in Q8_0 and MXFP4 with a router
bias of log Zipf(1.2) popularity + N(0, 0.5) (configs.zipf_router_bias).  At T = 4096 the routing
(ids and per-expert counts) is bit-exact with the oracle's, the hottest expert draws well over the
mean load, and the layer output (the tensor-core prefill path) is within the north-star tolerance
on sampled rows."""
import numpy as np
import pytest
import torch

from tests.helpers import C, U, bf16_bits_to_f32, oracle_desc, selected_host_weights, to_cuda_bf16, umsx, x_bits

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 5e-3, 2e-2


@pytest.mark.parametrize("name", ["qwen3-skew-q8_0", "qwen3-skew-mxfp4"])
def test_zipf_skew_layer_t4096(oracle, name):
    cfg = C.CONFIGS[name]
    T = 4096
    bias = umsx.configs.zipf_router_bias(cfg.experts, seed=cfg.seed)
    router = selected_host_weights(oracle, cfg, 0, [])
    router.router_b = bias
    layer = U.MoeLayer(cfg.desc(T), synthetic=cfg.synthetic())
    layer.set_router(router.router_w, bias)
    xb = x_bits(oracle, cfg, T, stream=0xFFFF9)
    x = to_cuda_bf16(xb)
    ids, wt, counts = layer.route(x)
    desc = oracle_desc(cfg)
    want_ids, want_w, _ = oracle.route(desc, router, bf16_bits_to_f32(xb))
    np.testing.assert_array_equal(ids.cpu().numpy(), want_ids)
    np.testing.assert_array_equal(wt.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    want_counts = np.bincount(want_ids.reshape(-1), minlength=cfg.experts)
    np.testing.assert_array_equal(counts.cpu().numpy(), want_counts)
    assert want_counts.max() > 8 * want_counts.mean(), want_counts.max() / want_counts.mean()
    out = layer.forward(x).cpu().numpy()
    rows = np.unique(np.linspace(0, T - 1, 96).astype(np.int64))
    w = selected_host_weights(oracle, cfg, 0, want_ids[rows])
    w.router_b = bias
    want = oracle.moe_layer(desc, w, bf16_bits_to_f32(xb[rows]), threads=16)
    err = out[rows].astype(np.float64) - want["out"].astype(np.float64)
    rel = np.linalg.norm(err) / np.linalg.norm(want["out"].astype(np.float64))
    scale = float(np.abs(want["out"]).max())
    assert rel <= REL_L2 and np.abs(err).max() <= MAX_ABS * max(1.0, scale), (rel, np.abs(err).max(), scale)
    layer.close()
