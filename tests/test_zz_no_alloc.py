"""umsx_route_static, the entry point for callers that cannot allocate device memory (needs a B200).

Such a caller (an operator inside a framework that pre-plans every buffer, or a process
whose device memory budget is spent) cannot create a layer handle.  umsx_route_static runs
the same router kernel with its scratch in a fixed array inside the library.  Its results
must equal umsx_route's bit for bit -- the tolerance every routing test here uses -- on two
calls in a row, which also shows the shared array is cleared between calls.  This file is
collected last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest

from tests.helpers import U, host_weights, small_config, weights_dict, x_bits

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _bf16(xb):
    return torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).cuda()


def _x(oracle, cfg, tokens, stream, dtype):
    xb = x_bits(oracle, cfg, tokens, stream=stream)
    if dtype == "bf16":
        return _bf16(xb)
    return torch.from_numpy((xb.astype(np.uint32) << 16).view(np.float32)).cuda()


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("routing", [U.ROUTE_TOPK_SOFTMAX, U.ROUTE_SOFTMAX_TOPK_NORM])
def test_route_static_equals_route_on_consecutive_calls(oracle, routing, dtype):
    cfg = small_config(routing=routing, experts=16, top_k=4, has_router_bias=routing == U.ROUTE_TOPK_SOFTMAX)
    w = host_weights(oracle, cfg)
    layer = U.MoeLayer(cfg.desc(64), weights_dict(w))
    rw = torch.from_numpy(w.router_w).cuda()
    rb = torch.from_numpy(w.router_b).cuda() if w.router_b is not None else None
    for tokens, stream in ((7, 0xFFFF0), (3, 0xFFFF1)):  # two calls in a row, different sizes and inputs
        x = _x(oracle, cfg, tokens, stream, dtype)
        ids_ref, w_ref, counts_ref = layer.route(x)
        ids, wt, counts = U.route_static(x, rw, rb, cfg.experts, cfg.top_k, cfg.routing, cfg.routed_scale)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
        np.testing.assert_array_equal(wt.cpu().numpy().view(np.uint32), w_ref.cpu().numpy().view(np.uint32))
        np.testing.assert_array_equal(counts.cpu().numpy(), counts_ref.cpu().numpy())
    layer.close()


def test_route_static_rejects_sizes_beyond_its_scratch(oracle):
    cfg = small_config()
    w = host_weights(oracle, cfg)
    rw = torch.from_numpy(w.router_w).cuda()
    x = _bf16(x_bits(oracle, cfg, 65))
    with pytest.raises(U.UmsxError) as e:
        U.route_static(x, rw, None, cfg.experts, cfg.top_k, cfg.routing)
    assert e.value.status == U.EINVAL and "tokens <= 64" in str(e.value)


def test_route_static_at_its_limits(oracle):
    """The largest request the fixed array holds (T = 64, E = 256, k = 8, H = 4096: the largest carve,
    and T * k = 512, the fused-dispatch bound) equals umsx_route bit for bit; H = 4160 is refused."""
    cfg = small_config(hidden=4096, intermediate=64, experts=256, top_k=8, routing=U.ROUTE_SOFTMAX_TOPK_NORM,
                       has_router_bias=True, has_bias=False, seed=31)
    w = host_weights(oracle, cfg)
    layer = U.MoeLayer(cfg.desc(64), weights_dict(w))
    rw = torch.from_numpy(w.router_w).cuda()
    rb = torch.from_numpy(w.router_b).cuda()
    for call in range(2):
        x = _x(oracle, cfg, 64, 0xFFFF2 + call, "f32")
        ids_ref, w_ref, counts_ref = layer.route(x)
        ids, wt, counts = U.route_static(x, rw, rb, cfg.experts, cfg.top_k, cfg.routing, cfg.routed_scale)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
        np.testing.assert_array_equal(wt.cpu().numpy().view(np.uint32), w_ref.cpu().numpy().view(np.uint32))
        np.testing.assert_array_equal(counts.cpu().numpy(), counts_ref.cpu().numpy())
    layer.close()
    wide = torch.zeros((4, 4160), dtype=torch.float32, device="cuda")
    with pytest.raises(U.UmsxError) as e:
        U.route_static(wide, torch.zeros((16, 4160), dtype=torch.float32, device="cuda"), None, 16, 4,
                       U.ROUTE_TOPK_SOFTMAX)
    assert e.value.status == U.EINVAL
