"""The host twins of the device generator (CPU only): drawing only the routed experts gives the
same blocks as drawing the whole layer, so the full-shape GPU tests check against the right weights."""
import numpy as np

from tests.helpers import C, host_weights, selected_host_weights, small_config


def test_selected_weights_equal_the_full_draw(oracle):
    for cfg in (small_config(), small_config(quant=8, fused_gate_up=False, has_bias=False, seed=5)):
        full = host_weights(oracle, cfg, layer=2)
        pick = [1, 5, 6]
        sel = selected_host_weights(oracle, cfg, 2, np.array([[5, 1], [6, 5]]))
        for name in ("gate_up", "gate", "up", "down"):
            a, b = getattr(full, name), getattr(sel, name)
            if a is None:
                assert b is None
                continue
            np.testing.assert_array_equal(a[pick], b[pick])
            assert not b[[e for e in range(cfg.experts) if e not in pick]].any()
        np.testing.assert_array_equal(full.router_w, sel.router_w)
        for name in ("router_b", "gate_up_bias", "down_bias"):
            a, b = getattr(full, name), getattr(sel, name)
            assert (a is None and b is None) or np.array_equal(a, b)
