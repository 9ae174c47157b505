"""Device status reporting (needs a B200): a non-finite combined output is rejected as the reference
rejects it (ExpertPlan, tools/engine/expert_dispatch.cpp:14-18, :84-85) -- UMSX_ENONFINITE from the
synchronous calls and from umsx_moe_status / umsx_stack_status after asynchronous ones -- on the
one-token kernel (T = 1), the per-stage kernels (T = 5) and the tensor-core prefill path (T = 80); the
record is cleared once read, and the same handle serves finite work afterwards."""
import numpy as np
import pytest
import torch

from tests.helpers import U, host_weights, small_config, umsx, weights_dict, x_bits

pytestmark = pytest.mark.gpu

BF16_INF = 0x7F80


def _layers(oracle, max_tokens):
    cfg = small_config()
    w = host_weights(oracle, cfg)
    good = U.MoeLayer(cfg.desc(max_tokens), weights_dict(w))
    bad_w = weights_dict(w)
    bad_w["down_bias"] = np.full_like(w.down_bias, BF16_INF)  # every expert's output row becomes +inf
    bad = U.MoeLayer(cfg.desc(max_tokens), bad_w)
    return cfg, good, bad


@pytest.mark.parametrize("tokens", [1, 5, 80])
def test_nonfinite_layer_output_is_rejected(oracle, tokens):
    cfg, good, bad = _layers(oracle, tokens)
    xb = x_bits(oracle, cfg, tokens)
    xh = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16)
    oh = torch.empty((tokens, cfg.hidden), dtype=torch.float32)
    with pytest.raises(U.UmsxError) as e:
        bad.forward_host(xh, oh)
    assert e.value.status == U.ENONFINITE
    assert np.isinf(oh.numpy()).all()
    # asynchronous call, then the status query; the record is cleared once read
    bad.forward(xh.cuda())
    with pytest.raises(U.UmsxError) as e:
        bad.status()
    assert e.value.status == U.ENONFINITE
    bad.status()
    good.forward_host(xh, oh)
    assert np.isfinite(oh.numpy()).all()
    good.status()
    good.close()
    bad.close()


@pytest.mark.parametrize("tokens", [1, 5])
def test_nonfinite_stack_output_is_rejected(oracle, tokens):
    cfg, good, bad = _layers(oracle, 8)
    stack = umsx.MoeStack([good, bad, good], max_tokens=8)
    xb = x_bits(oracle, cfg, tokens)
    xh = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).pin_memory()
    oh = torch.empty((tokens, cfg.hidden), dtype=torch.float32).pin_memory()
    with pytest.raises(U.UmsxError) as e:
        stack.forward_host(xh, oh)
    assert e.value.status == U.ENONFINITE
    stack.forward(xh.cuda())
    with pytest.raises(U.UmsxError) as e:
        stack.status()
    assert e.value.status == U.ENONFINITE
    stack.status()
    stack.close()
    good.close()
    bad.close()


@pytest.mark.parametrize("tokens", [1, 3])
def test_bounded_grid_wait_runs_out_and_the_stack_recovers(oracle, tokens):
    """A CTA of the one-launch decode kernel withholds its first grid-barrier arrival (a flag that
    nothing else sets): every other CTA's bounded wait runs out (about 1 ms here), the kernel ends,
    the call reports UMSX_ETIMEOUT, and the next forward on the same stack gives the usual bits.
    T = 1 runs the one-token kernel, T = 3 the multi-token kernel."""
    cfg = small_config()
    layers = [U.MoeLayer(cfg.desc(4), synthetic=cfg.synthetic(layer=l)) for l in range(3)]
    stack = umsx.MoeStack(layers, max_tokens=4)
    xb = x_bits(oracle, cfg, tokens)
    xh = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).pin_memory()
    want = torch.empty((tokens, cfg.hidden), dtype=torch.float32).pin_memory()
    stack.forward_host(xh, want)
    want = want.numpy().copy()
    oh = torch.empty((tokens, cfg.hidden), dtype=torch.float32).pin_memory()
    stack.inject_fault(cta=5, wait_limit_cycles=2_000_000)
    with pytest.raises(U.UmsxError) as e:
        stack.forward_host(xh, oh)
    assert e.value.status == U.ETIMEOUT
    stack.forward_host(xh, oh)
    np.testing.assert_array_equal(oh.numpy().view(np.uint32), want.view(np.uint32))
    # asynchronous form: the status query reports it
    stack.inject_fault(cta=0, wait_limit_cycles=2_000_000)
    stack.forward(xh.cuda())
    with pytest.raises(U.UmsxError) as e:
        stack.status()
    assert e.value.status == U.ETIMEOUT
    got = stack.forward(xh.cuda()).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    stack.close()
    for l in layers:
        l.close()
