"""Expert-residency admission policy (CPU): the product's policy (umsx_bank_simulate, the same code the
banked layers run) against the restatement of the reference's rules in oracle/bank.py, on
hand-derived known answers and on seeded random dispatch sequences."""
import numpy as np
import pytest

from oracle.bank import LFU, LRU, RefBank
from tests.helpers import U


def ref_run(experts, slots, policy, dispatches):
    b = RefBank(experts, slots, policy)
    return [b.dispatch(list(sel), admit) for sel, admit in dispatches], b.stats


def test_lru_known_answer():
    # hybrid patch :3138-3145: a miss takes a free slot, else the least recently used resident that
    # this dispatch did not select; batches (admit False) look up only.
    d = [([0, 1], True), ([2, 0], True), ([3, 2], False), ([3], True)]
    slots, st = U.bank_simulate(8, 2, U.BANK_LRU, d)
    assert slots == [[0, 1], [1, 0], [-1, 1], [0]]
    assert {k: st[k] for k in ("dispatches", "demands", "hits", "misses", "admissions", "evictions", "transient")} == \
        dict(dispatches=4, demands=7, hits=2, misses=5, admissions=4, evictions=2, transient=1)
    assert (slots, {k: v for k, v in st.items() if k != "upload_bytes"}) == \
        (ref_run(8, 2, LRU, d)[0], {k: v for k, v in ref_run(8, 2, LRU, d)[1].items() if k != "upload_bytes"})


def test_lfu_known_answer():
    # :3091-3101 / :3121-3137: one demand fills a free slot; replacing a resident needs 6 demands
    # (and a strictly higher count); the demand window halves every count after about 2.45 bank-fulls.
    d = [([0, 1], True), ([2, 3], True), ([2, 3], True)]
    slots, st = U.bank_simulate(8, 2, U.BANK_LFU, d)
    assert slots == [[0, 1], [-1, -1], [-1, -1]]
    assert st["admissions"] == 2 and st["evictions"] == 0 and st["transient"] == 4 and st["halvings"] == 1


def test_lfu_insert_cap_and_lru_without_cap():
    d = [([0, 1, 2, 3, 4, 5], True)]
    assert U.bank_simulate(16, 8, U.BANK_LFU, d)[0] == [[0, 1, 2, 3, -1, -1]]
    assert U.bank_simulate(16, 8, U.BANK_LRU, d)[0] == [[0, 1, 2, 3, 4, 5]]


def test_lfu_hot_expert_replaces_cold_resident():
    # a single-slot bank: expert 0 takes the free slot; expert 1, demanded every dispatch after it,
    # replaces it once its count reaches 6 (counts of expert 1 after each dispatch, halvings included:
    # 1 1 2 3 2 3 4 5 3 4 5 6), at the 13th dispatch
    d = [([0], True)] + [([1], True)] * 12
    slots, st = U.bank_simulate(4, 1, U.BANK_LFU, d)
    assert slots == [[0]] + [[-1]] * 11 + [[0]]
    assert st["evictions"] == 1 and st["halvings"] == 3
    assert slots == ref_run(4, 1, LFU, d)[0]


def _random_sequence(rng, experts, top_k, n, batch_every, skew):
    p = rng.zipf(skew, size=experts * 4) % experts if skew else None
    seq = []
    for i in range(n):
        if batch_every and i % batch_every == batch_every - 1:
            t = int(rng.integers(2, 9))
            ids = [list(rng.choice(experts, size=top_k, replace=False)) for _ in range(t)]
            seen, sel = set(), []
            for row in ids:
                for e in row:
                    if e not in seen:
                        seen.add(e)
                        sel.append(int(e))
            seq.append((sel, False))
        else:
            if p is not None:
                cand = list(dict.fromkeys(int(e) for e in rng.choice(p, size=4 * top_k)))
                extra = [int(e) for e in rng.permutation(experts) if e not in cand]
                sel = (cand + extra)[:top_k]
            else:
                sel = [int(e) for e in rng.choice(experts, size=top_k, replace=False)]
            seq.append((sel, True))
    return seq


@pytest.mark.parametrize("policy", [LFU, LRU])
@pytest.mark.parametrize("experts,top_k,slots,skew", [(32, 4, 8, None), (32, 4, 8, 1.3), (128, 4, 32, 1.2),
                                                      (64, 6, 16, 1.5), (16, 2, 1, None), (16, 4, 16, 1.2)])
def test_policy_matches_restatement(policy, experts, top_k, slots, skew):
    rng = np.random.default_rng(experts * 131 + top_k * 7 + slots + policy)
    seq = _random_sequence(rng, experts, top_k, 400, 7, skew)
    got, st = U.bank_simulate(experts, slots, policy, seq)
    want, wst = ref_run(experts, slots, policy, seq)
    assert got == want
    for k in ("dispatches", "demands", "hits", "misses", "admissions", "evictions", "transient", "halvings"):
        assert st[k] == wst[k], k
    # invariants: no two selected experts of a dispatch share a slot; hits + misses = demands
    for row in got:
        resident = [s for s in row if s >= 0]
        assert len(resident) == len(set(resident)) and all(s < slots for s in resident)
    assert st["hits"] + st["misses"] == st["demands"]


def test_simulate_rejects_bad_arguments():
    with pytest.raises(U.UmsxError):
        U.bank_simulate(8, 9, U.BANK_LRU, [([0], True)])
    with pytest.raises(U.UmsxError):
        U.bank_simulate(8, 2, 7, [([0], True)])
    with pytest.raises(U.UmsxError):
        U.bank_simulate(8, 2, U.BANK_LFU, [([8], True)])
    with pytest.raises(U.UmsxError):
        U.bank_simulate(8, 2, U.BANK_LFU, [([], True)])


def test_create_banked_rejects_bad_arguments(oracle):
    """Argument checks of umsx_moe_create_banked run before any device call (CPU)."""
    from tests.helpers import host_weights, small_config, weights_dict
    cfg = small_config(experts=8, top_k=2)
    wd = weights_dict(host_weights(oracle, cfg))
    for bank in ((0, U.BANK_LFU), (9, U.BANK_LRU), (4, 5)):
        with pytest.raises(U.UmsxError) as e:
            U.MoeLayer(cfg.desc(4), wd, bank=bank)
        assert e.value.status == U.EINVAL
    with pytest.raises(U.UmsxError) as e:
        U.MoeLayer(cfg.desc(4, ep_rank=0, ep_world=2), wd, bank=(2, U.BANK_LFU))
    assert e.value.status == U.EINVAL
