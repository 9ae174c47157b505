"""Banked layers (umsx_moe_create_banked) on the GPU: every call's output is bit-identical to the
resident layer's on the same weights, whatever the bank holds at the time, and the bank's counters and
residency follow the policy restated from the reference (oracle/bank.py) over the same routing."""
import numpy as np
import pytest

from oracle.bank import RefBank
from tests.helpers import U, bits, host_weights, small_config, to_cuda_bf16, weights_dict, x_bits

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

STATS = ("dispatches", "demands", "hits", "misses", "admissions", "evictions", "transient", "halvings")


def _cfg(which):
    if which == "mxfp4":
        return small_config(experts=32, top_k=4, seed=21)
    return small_config(name="small-q8", quant=U.QUANT_Q8_0, routing=U.ROUTE_SOFTMAX_TOPK_NORM,
                        activation=U.ACT_SILU, fused_gate_up=False, has_bias=False, has_router_bias=False,
                        experts=16, top_k=4, seed=12)


def _distinct(ids):
    seen, sel = set(), []
    for e in ids.reshape(-1).tolist():
        if e not in seen:
            seen.add(e)
            sel.append(e)
    return sel


@pytest.mark.parametrize("policy", [U.BANK_LFU, U.BANK_LRU])
@pytest.mark.parametrize("which", ["mxfp4", "q8_0"])
def test_banked_layer_matches_resident(oracle, policy, which):
    cfg = _cfg(which)
    K, E, n_slots = cfg.top_k, cfg.experts, 6
    wd = weights_dict(host_weights(oracle, cfg))
    res = U.MoeLayer(cfg.desc(64), wd)
    bank = U.MoeLayer(cfg.desc(64), wd, bank=(n_slots, policy))
    ref = RefBank(E, n_slots, policy)
    # one-token calls over a few repeating token streams (reuse the bank can exploit), batches between
    seq = [1] * 24 + [5] + [1] * 10 + [40] + [1] * 10 + [64] + [1] * 4
    for i, T in enumerate(seq):
        stream = 0xB000 + (i % 5 if T == 1 else 100 + i)
        x = to_cuda_bf16(x_bits(oracle, cfg, T, stream=stream))
        ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
        want = res.forward(x, ids=ids)
        got = bank.forward(x)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bits(got.cpu().numpy()), bits(want.cpu().numpy()), err_msg=f"call {i} T={T}")
        ids_h = ids.cpu().numpy()
        ref.dispatch(ids_h[0].tolist() if T == 1 else _distinct(ids_h), T == 1)
    st = bank.bank_stats()
    for k in STATS:
        assert st[k] == ref.stats[k], k
    np.testing.assert_array_equal(st["slot_of_expert"], np.array(ref.slot_map, np.int32))
    per_expert = 3 * cfg.intermediate * (cfg.hidden // 32) * U.BLOCK_BYTES[cfg.quant]
    assert st["upload_bytes"] == (st["admissions"] + st["transient"]) * per_expert
    assert st["hits"] > 0 and st["admissions"] > 0
    res.close()
    bank.close()


def test_banked_layer_host_buffers_and_refusals(oracle):
    cfg = _cfg("mxfp4")
    wd = weights_dict(host_weights(oracle, cfg))
    res = U.MoeLayer(cfg.desc(8), wd)
    bank = U.MoeLayer(cfg.desc(8), wd, bank=(4, U.BANK_LFU))
    for i, T in enumerate([1, 1, 3, 1, 8, 1]):
        xb = x_bits(oracle, cfg, T, stream=0xC000 + i % 2)
        x_host = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).pin_memory()
        a = torch.empty((T, cfg.hidden), dtype=torch.float32).pin_memory()
        b = torch.empty((T, cfg.hidden), dtype=torch.float32).pin_memory()
        res.forward_host(x_host, a)
        bank.forward_host(x_host, b)
        np.testing.assert_array_equal(bits(b.numpy()), bits(a.numpy()), err_msg=f"call {i}")
    x = to_cuda_bf16(x_bits(oracle, cfg, 2))
    for call in (lambda: bank.forward_jobs(x), lambda: bank.export_expert(U.PROJ_DOWN, 0),
                 lambda: U.MoeStack([bank], 4, 1e-5)):
        with pytest.raises(U.UmsxError) as e:
            call()
        assert e.value.status == U.EUNSUPPORTED
    res.close()
    bank.close()
