"""CUDA path vs the CPU oracle and the reference golden vectors, through the C ABI (needs a B200).

Bar: bit-exact for ids, counts, dequantised weights, the MXFP4 x Q8_0 and Q8_0 x Q8_0
dots, and (because every fp32 step shares its order with the oracle) the layer output.
"""
import os

import numpy as np
import pytest

from tests.helpers import (U, bf16_bits_to_f32, bits, host_weights, oracle_desc, small_config, to_cuda_bf16,
                           weights_dict, x_bits)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def down_only_layer(down_blocks, hidden, inter, experts, quant=U.QUANT_MXFP4, down_bias=None):
    """A handle whose down projection is the given ggml blocks (other tensors zero)."""
    bb = U.BLOCK_BYTES[quant]
    w = dict(router_w=np.zeros((experts, hidden), np.float32),
             gate_up=np.zeros((experts, 2 * inter, hidden // 32 * bb), np.uint8),
             down=np.ascontiguousarray(down_blocks, np.uint8).reshape(experts, hidden, inter // 32 * bb))
    has_bias = down_bias is not None
    if has_bias:
        w["gate_up_bias"] = np.zeros((experts, 2 * inter), np.uint16)
        w["down_bias"] = down_bias
    d = U.Desc(hidden, inter, experts, 1, quant, U.ROUTE_TOPK_SOFTMAX, U.ACT_SWIGLU_OAI, 1, int(has_bias), 0,
               1.702, 7.0, 1.0, 64, 0, 1)
    return U.MoeLayer(d, w)


def test_down_golden_quantized_cuda_cases():
    """tests/test_quantized_cuda.cpp:31-41 samples, bitwise vs the reference's vec_dot."""
    g = np.load(os.path.join(GOLD, "quantized_down.npz"))
    layer = down_only_layer(g["weights"], 64, 128, 3)
    experts = g["jobs"][:, 2].astype(np.int32)
    for s in range(12):
        got = layer.expert_down_q8(torch.from_numpy(g[f"s{s}_act"]).cuda(), experts).cpu().numpy()
        np.testing.assert_array_equal(bits(got), bits(g[f"s{s}_out"]), err_msg=f"sample {s}")
    with pytest.raises(U.UmsxError) as e:
        layer.expert_down_q8(torch.zeros((1, 4 * 34), dtype=torch.uint8, device="cuda"), np.array([3], np.int32))
    assert e.value.status == U.ENOTRESIDENT
    layer.close()


def test_down_golden_adversarial_bank():
    """hybrid_layer.cpp:964-979 bank (E8M0 0/1/2/120/126/127/128/130, all codes) x sine/zero/q8-ties."""
    g = np.load(os.path.join(GOLD, "compatible_down.npz"))
    layer = down_only_layer(g["weights"], 64, 128, 4)
    for pattern in ("sine", "zero", "q8-ties"):
        for sample in range(3):
            act = g[f"{pattern}_{sample}_act"]
            experts = (np.arange(act.shape[0]) % 4).astype(np.int32)
            got = layer.expert_down_q8(torch.from_numpy(act).cuda(), experts).cpu().numpy()
            np.testing.assert_array_equal(bits(got), bits(g[f"{pattern}_{sample}_out"]), err_msg=f"{pattern} {sample}")
    layer.close()


def test_down_golden_exact_packed_417():
    """tests/test_exact_packed_cpu.cpp cases (seed 417), rows padded to 64 with zero blocks."""
    from tests.golden.make_golden import exact_packed_inputs
    from oracle.oracle import Oracle
    orc = Oracle()
    g = np.load(os.path.join(GOLD, "exact_packed_417.npz"))
    for n, columns, w, floats in exact_packed_inputs():
        timing = columns < 0
        columns = abs(columns)
        nb = n // 32
        rows = max(64, (columns + 63) // 64 * 64)
        blocks = np.zeros((rows * nb, 17), np.uint8)
        blocks[:columns * nb] = w
        layer = down_only_layer(blocks, rows, n, 1)
        if timing:
            act = orc.quantize_q8_0(floats)[None, :]
            exp = g["timing_gemv_2880"]
        else:
            act = orc.quantize_q8_0(floats.reshape(8, n))[:1].copy()
            act.reshape(-1)[2] = 0x80
            exp = g[f"gemv_{n}_{columns}"]
        got = layer.expert_down_q8(torch.from_numpy(act).cuda(), np.zeros(1, np.int32)).cpu().numpy()[0, :columns]
        np.testing.assert_array_equal(bits(got), bits(exp), err_msg=f"n={n} columns={columns}")
        if not timing:
            acts = orc.quantize_q8_0(floats.reshape(8, n))
            got = layer.expert_down_q8(torch.from_numpy(acts).cuda(), np.zeros(8, np.int32)).cpu().numpy()
            for rws in (4, 8):
                stride = columns + 3
                exp = g[f"gemm_{n}_{columns}_{rws}"].reshape(rws, stride)
                np.testing.assert_array_equal(bits(got[:rws, :columns]), bits(exp[:, :columns]))
        layer.close()


@pytest.mark.parametrize("quant", [U.QUANT_MXFP4, U.QUANT_Q8_0])
def test_repack_export_round_trip(oracle, quant):
    cfg = small_config(quant=quant, fused_gate_up=quant == U.QUANT_MXFP4, has_bias=quant == U.QUANT_MXFP4)
    w = host_weights(oracle, cfg)
    layer = U.MoeLayer(cfg.desc(8), weights_dict(w))
    syn = U.MoeLayer(cfg.desc(8), synthetic=cfg.synthetic())
    for e in range(cfg.experts):
        if cfg.fused_gate_up:
            np.testing.assert_array_equal(layer.export_expert(U.PROJ_GATE_UP, e), w.gate_up[e].reshape(-1))
            np.testing.assert_array_equal(syn.export_expert(U.PROJ_GATE_UP, e), w.gate_up[e].reshape(-1))
        else:
            np.testing.assert_array_equal(layer.export_expert(U.PROJ_GATE, e), w.gate[e].reshape(-1))
            np.testing.assert_array_equal(syn.export_expert(U.PROJ_UP, e), w.up[e].reshape(-1))
        np.testing.assert_array_equal(syn.export_expert(U.PROJ_DOWN, e), w.down[e].reshape(-1))
    with pytest.raises(U.UmsxError):
        layer.export_expert(U.PROJ_DOWN, cfg.experts)
    layer.close()
    syn.close()


def _layer_case(oracle, cfg, tokens, synthetic=True, x_dtype="bf16"):
    w = host_weights(oracle, cfg)
    xb = x_bits(oracle, cfg, tokens)
    x32 = bf16_bits_to_f32(xb)
    want = oracle.moe_layer(oracle_desc(cfg), w, x32, threads=8)
    layer = U.MoeLayer(cfg.desc(max(tokens, 4)), synthetic=cfg.synthetic()) if synthetic else \
        U.MoeLayer(cfg.desc(max(tokens, 4)), weights_dict(w))
    x = to_cuda_bf16(xb) if x_dtype == "bf16" else torch.from_numpy(x32).cuda()
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int32, device="cuda")
    wt = torch.empty((tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    out = layer.forward(x, ids=ids, weights=wt).cpu().numpy()
    torch.cuda.synchronize()
    return layer, want, out, ids.cpu().numpy(), wt.cpu().numpy(), x


@pytest.mark.parametrize("tokens", [1, 3, 16, 40])
def test_layer_mxfp4_bit_exact(oracle, tokens):
    cfg = small_config()
    layer, want, out, ids, wt, x = _layer_case(oracle, cfg, tokens)
    np.testing.assert_array_equal(ids, want["ids"])
    np.testing.assert_array_equal(bits(wt), bits(want["weights"]))
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    r_ids, r_w, counts = layer.route(x)
    np.testing.assert_array_equal(r_ids.cpu().numpy(), want["ids"])
    np.testing.assert_array_equal(counts.cpu().numpy(), want["counts"])
    layer.close()


@pytest.mark.parametrize("tokens", [1, 5, 33])
def test_layer_q8_0_bit_exact(oracle, tokens):
    cfg = small_config(name="small-q8", quant=U.QUANT_Q8_0, routing=U.ROUTE_SOFTMAX_TOPK_NORM, activation=U.ACT_SILU,
                       fused_gate_up=False, has_bias=False, has_router_bias=False, experts=16, top_k=4, seed=12)
    layer, want, out, ids, wt, x = _layer_case(oracle, cfg, tokens, synthetic=False, x_dtype="f32")
    np.testing.assert_array_equal(ids, want["ids"])
    np.testing.assert_array_equal(bits(wt), bits(want["weights"]))
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    layer.close()


def test_layer_deepseek_routing_bit_exact(oracle):
    cfg = small_config(name="small-ds", quant=U.QUANT_Q8_0, routing=U.ROUTE_SOFTMAX_TOPK, activation=U.ACT_SILU,
                       fused_gate_up=False, has_bias=False, has_router_bias=False, experts=16, top_k=6, seed=14)
    layer, want, out, ids, wt, _ = _layer_case(oracle, cfg, 7)
    np.testing.assert_array_equal(ids, want["ids"])
    np.testing.assert_array_equal(bits(out), bits(want["out"]))
    layer.close()


def test_route_ties_go_to_the_lowest_index(oracle):
    """Equal logits everywhere: top-k must be experts 0..k-1 (topk-tie-probe.cpp:111-113)."""
    cfg = small_config(has_router_bias=False)
    w = host_weights(oracle, cfg)
    w.router_w[:] = 0.0
    w.router_w[5] = 0.0
    layer = U.MoeLayer(cfg.desc(8), weights_dict(w))
    x = to_cuda_bf16(x_bits(oracle, cfg, 4))
    ids, wt, counts = layer.route(x)
    assert (ids.cpu().numpy() == np.arange(cfg.top_k)[None, :]).all()
    assert np.allclose(wt.cpu().numpy(), 1.0 / cfg.top_k)
    # pairwise ties: duplicated rows give equal logits; lower index must win
    w.router_w[:] = w.router_w[0]
    w.router_w[3] = w.router_w[0] * 2
    w.router_w[6] = w.router_w[0] * 2
    layer2 = U.MoeLayer(cfg.desc(8), weights_dict(w))
    xb = x_bits(oracle, cfg, 4)
    ids2, _, _ = layer2.route(to_cuda_bf16(xb))
    want_ids, _, _ = oracle.route(oracle_desc(cfg), w, bf16_bits_to_f32(xb))
    np.testing.assert_array_equal(ids2.cpu().numpy(), want_ids)
    layer.close()
    layer2.close()


def test_mul_mat_id_masked_rows(oracle):
    """-1 ids give exact-zero rows, other rows equal the oracle (tests/test_masked_matmul.cpp)."""
    cfg = small_config()
    w = host_weights(oracle, cfg)
    layer = U.MoeLayer(cfg.desc(8), weights_dict(w))
    T, n_ids = 4, 3
    rng = np.random.default_rng(5)
    b = rng.standard_normal((T, 1, cfg.hidden)).astype(np.float32)
    ids = np.array([[0, -1, 3], [7, 2, -1], [-1, -1, -1], [5, 6, 1]], np.int32)
    dst = layer.mul_mat_id(U.PROJ_GATE_UP, torch.from_numpy(b).cuda(), torch.from_numpy(ids).cuda()).cpu().numpy()
    for t in range(T):
        a = oracle.quantize_q8_0(b[t, 0])
        for i in range(n_ids):
            if ids[t, i] < 0:
                assert np.all(bits(dst[t, i]) == 0)
            else:
                exp = oracle.gemv(U.QUANT_MXFP4, cfg.hidden, w.gate_up[ids[t, i]], a)
                np.testing.assert_array_equal(bits(dst[t, i]), bits(exp))
    layer.close()


def test_combine_rank_order():
    """1e20 - 1e20 + 1 == 1 only in rank order (tests/test_expert_dispatch.cpp:65-73)."""
    y = torch.tensor([[[1e20] * 4, [-1e20] * 4, [1.0] * 4]], dtype=torch.float32, device="cuda")
    w = torch.ones((1, 3), dtype=torch.float32, device="cuda")
    out = U.combine(y, w).cpu().numpy()
    assert (out == 1.0).all()


def test_full_size_gpt_oss_20b_layer(oracle):
    """configs[0] at full size, T in {1, 32}: bit-exact against the oracle."""
    from tests.helpers import C
    cfg = C.GPT_OSS_20B
    for tokens in (1, 32):
        layer, want, out, ids, wt, _ = _layer_case(oracle, cfg, tokens)
        np.testing.assert_array_equal(ids, want["ids"])
        np.testing.assert_array_equal(bits(out), bits(want["out"]))
        layer.close()


def test_stack_rmsnorm_residual_bit_exact(oracle):
    """h <- h + MoE_l(RMSNorm(h)) over 3 layers (configs[2] structure, small shapes), graph replay."""
    from tests.helpers import umsx
    cfg = small_config()
    L, T = 3, 5
    layers = [U.MoeLayer(cfg.desc(1), synthetic=cfg.synthetic(layer=l)) for l in range(L)]
    stack = umsx.MoeStack(layers, max_tokens=8)
    xb = x_bits(oracle, cfg, T)
    h = bf16_bits_to_f32(xb).copy()
    for l in range(L):
        xn = oracle.rmsnorm(h, 1e-5)
        h = (h + oracle.moe_layer(oracle_desc(cfg), host_weights(oracle, cfg, layer=l), xn, threads=8)["out"])
        h = h.astype(np.float32)
    x = to_cuda_bf16(xb)
    for _ in range(2):  # capture, then replay
        got = stack.forward(x).cpu().numpy()
        np.testing.assert_array_equal(bits(got), bits(h))
    hostout = torch.empty((T, cfg.hidden), dtype=torch.float32).pin_memory()
    stack.forward_host(torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).pin_memory(), hostout)
    np.testing.assert_array_equal(bits(hostout.numpy()), bits(h))
    stack.set_timing(True)
    stack.forward(x)
    st = stack.stage_times()
    assert all(v > 0 for v in st.values()), st
    stack.close()
    for l in layers:
        l.close()
