"""Test helpers: host twins of the synthetic weights, oracle descriptors, small configs."""
from __future__ import annotations

import dataclasses

import numpy as np

from __graft_entry__ import load_package
from oracle.oracle import LayerWeights, OrcDesc

umsx = load_package()
C = umsx.configs
U = umsx.umsx


def oracle_desc(cfg) -> OrcDesc:
    return OrcDesc(cfg.hidden, cfg.intermediate, cfg.experts, cfg.top_k, cfg.quant, cfg.routing, cfg.activation,
                   int(cfg.fused_gate_up), int(cfg.has_bias), cfg.swiglu_alpha, cfg.swiglu_limit, cfg.routed_scale)


def host_weights(orc, cfg, layer: int = 0) -> LayerWeights:
    """The same tensors umsx_moe_create_synthetic draws on the device, drawn here by the oracle."""
    E, H, I = cfg.experts, cfg.hidden, cfg.intermediate
    s = cfg.seed
    sid = C.stream_id
    bb = U.BLOCK_BYTES[cfg.quant]

    def blocks(kind, n):
        if cfg.quant == U.QUANT_MXFP4:
            return orc.gen_mxfp4(s, sid(layer, kind), 0, n, 119, 5)
        return orc.gen_q8_0(s, sid(layer, kind), 0, n)

    router_w = orc.gen_normal_f32(s, sid(layer, C.KIND_ROUTER_W), 0, E * H, cfg.router_sigma).reshape(E, H)
    router_b = orc.gen_normal_f32(s, sid(layer, C.KIND_ROUTER_B), 0, E, cfg.router_bias_sigma) \
        if cfg.has_router_bias else None
    gate_up = gate = up = None
    if cfg.fused_gate_up:
        gate_up = blocks(C.KIND_GATE_UP, E * 2 * I * (H // 32)).reshape(E, 2 * I, H // 32 * bb)
    else:
        gate = blocks(C.KIND_GATE_UP, E * I * (H // 32)).reshape(E, I, H // 32 * bb)
        up = blocks(C.KIND_UP, E * I * (H // 32)).reshape(E, I, H // 32 * bb)
    down = blocks(C.KIND_DOWN, E * H * (I // 32)).reshape(E, H, I // 32 * bb)
    gub = db = None
    if cfg.has_bias:
        gub = orc.gen_normal_bf16(s, sid(layer, C.KIND_GU_BIAS), 0, E * 2 * I, cfg.bias_sigma).reshape(E, 2 * I)
        db = orc.gen_normal_bf16(s, sid(layer, C.KIND_DOWN_BIAS), 0, E * H, cfg.bias_sigma).reshape(E, H)
    return LayerWeights(router_w, router_b, gate_up, gate, up, down, gub, db)


def weights_dict(w: LayerWeights) -> dict:
    return {k: getattr(w, k) for k in ("router_w", "router_b", "gate_up", "gate", "up", "down", "gate_up_bias",
                                       "down_bias")}


def small_config(**over):
    """A gpt-oss-shaped layer shrunk so the oracle finishes in milliseconds."""
    base = dataclasses.replace(C.GPT_OSS_20B, name="small-mxfp4", hidden=256, intermediate=192, experts=8, top_k=2,
                               seed=11)
    return dataclasses.replace(base, **over)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def x_bits(orc, cfg, tokens: int, stream: int = 0xFFFF0, sigma: float = 1.0) -> np.ndarray:
    return orc.gen_normal_bf16(cfg.seed, stream, 0, tokens * cfg.hidden, sigma).reshape(tokens, cfg.hidden)


def bits(a) -> np.ndarray:
    """fp32 values as their bit patterns (bit-exact comparisons)."""
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def to_cuda_bf16(xb: np.ndarray):
    """bf16 bit patterns (uint16) -> a bf16 CUDA tensor."""
    import torch
    return torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).cuda()


def write_layer_gguf(paths, layer: int, w: LayerWeights, quant: int, hidden: int, inter: int, split_at: int = 99,
                     bias_dtype=np.float32, extra_kv: bool = True):
    """Writes one layer's router and expert tensors in llama.cpp's GGUF naming
    (blk.L.ffn_gate_inp.*, blk.L.ffn_{gate,up,down}_exps.*) with gguf-py.  `paths` lists the
    shard files; tensors after the first `split_at` go to the second shard.  Fused gate_up
    weights are written as the separate gate and up tensors a GGUF checkpoint holds."""
    import gguf
    qt = gguf.GGMLQuantizationType.MXFP4 if quant == U.QUANT_MXFP4 else gguf.GGMLQuantizationType.Q8_0
    pre = f"blk.{layer}."
    gate, up = (w.gate, w.up) if w.gate_up is None else (w.gate_up[:, :inter], w.gate_up[:, inter:])
    tensors = [(pre + "ffn_gate_inp.weight", np.ascontiguousarray(w.router_w, np.float32), None)]
    if w.router_b is not None:
        tensors.append((pre + "ffn_gate_inp.bias", np.ascontiguousarray(w.router_b, np.float32), None))
    tensors += [(pre + "ffn_gate_exps.weight", np.ascontiguousarray(gate, np.uint8), qt),
                (pre + "ffn_up_exps.weight", np.ascontiguousarray(up, np.uint8), qt),
                (pre + "ffn_down_exps.weight", np.ascontiguousarray(w.down, np.uint8), qt)]
    if w.gate_up_bias is not None:
        gb = bf16_bits_to_f32(w.gate_up_bias)
        tensors += [(pre + "ffn_gate_exps.bias", np.ascontiguousarray(gb[:, :inter]).astype(bias_dtype), None),
                    (pre + "ffn_up_exps.bias", np.ascontiguousarray(gb[:, inter:]).astype(bias_dtype), None),
                    (pre + "ffn_down_exps.bias", bf16_bits_to_f32(w.down_bias).astype(bias_dtype), None)]
    groups = [tensors[:split_at], tensors[split_at:]] if len(paths) > 1 else [tensors]
    for path, group in zip(paths, groups):
        wr = gguf.GGUFWriter(path, "gpt-oss")
        if extra_kv:
            wr.add_string("general.name", "umsx test layer")
            wr.add_uint32("test.count", 7)
            wr.add_array("test.list", [1, 2, 3])
            wr.add_array("test.names", ["a", "bc"])
            wr.add_float32("test.f", 0.5)
        for name, arr, raw in group:
            if raw is None:
                wr.add_tensor(name, arr)
            else:
                wr.add_tensor(name, arr, raw_dtype=raw)
        wr.write_header_to_file()
        wr.write_kv_data_to_file()
        wr.write_tensors_to_file()
        wr.close()


def selected_host_weights(orc, cfg, layer: int, experts) -> LayerWeights:
    """host_weights with only the listed experts' blocks drawn (the others stay zero): enough for the
    oracle, which reads only the experts its routing selects, at full BASELINE shapes."""
    E, H, I = cfg.experts, cfg.hidden, cfg.intermediate
    s, sid = cfg.seed, C.stream_id
    bb = U.BLOCK_BYTES[cfg.quant]

    def blocks(kind, rows, cols):
        out = np.zeros((E, rows, cols // 32 * bb), np.uint8)
        per = rows * (cols // 32)
        for e in sorted({int(v) for v in np.asarray(experts).reshape(-1)}):
            orc.gen_blocks_into(cfg.quant, out[e], s, sid(layer, kind), e * per, per, threads=8)
        return out

    router_w = orc.gen_normal_f32(s, sid(layer, C.KIND_ROUTER_W), 0, E * H, cfg.router_sigma).reshape(E, H)
    router_b = orc.gen_normal_f32(s, sid(layer, C.KIND_ROUTER_B), 0, E, cfg.router_bias_sigma) \
        if cfg.has_router_bias else None
    gate_up = gate = up = None
    if cfg.fused_gate_up:
        gate_up = blocks(C.KIND_GATE_UP, 2 * I, H)
    else:
        gate, up = blocks(C.KIND_GATE_UP, I, H), blocks(C.KIND_UP, I, H)
    down = blocks(C.KIND_DOWN, H, I)
    gub = db = None
    if cfg.has_bias:
        gub = orc.gen_normal_bf16(s, sid(layer, C.KIND_GU_BIAS), 0, E * 2 * I, cfg.bias_sigma).reshape(E, 2 * I)
        db = orc.gen_normal_bf16(s, sid(layer, C.KIND_DOWN_BIAS), 0, E * H, cfg.bias_sigma).reshape(E, H)
    return LayerWeights(router_w, router_b, gate_up, gate, up, down, gub, db)


def oracle_stack(orc, cfg, xb: np.ndarray, n_layers: int, threads: int = 16, eps: float = 1e-5) -> np.ndarray:
    """h <- h + MoE_l(RMSNorm(h)) on the oracle at full shapes, drawing only the routed experts."""
    h = bf16_bits_to_f32(xb).copy()
    desc = oracle_desc(cfg)
    for l in range(n_layers):
        xn = orc.rmsnorm(h, eps)
        router = selected_host_weights(orc, cfg, l, [])
        ids, _, _ = orc.route(desc, router, xn)
        w = selected_host_weights(orc, cfg, l, ids)
        h = (h + orc.moe_layer(desc, w, xn, threads=threads)["out"]).astype(np.float32)
    return h


def oracle_mixed_stack(orc, xb: np.ndarray, n_layers: int, threads: int = 16, eps: float = 1e-5,
                       first: int = 0) -> np.ndarray:
    """configs[4] block on the oracle: layer 0 the dense FFN, then h <- h + ((routed) + (shared FFN))
    per layer (the graph's ggml_add of the shared branch to the routed sum, then the residual);
    layers first .. first + n_layers - 1."""
    h = bf16_bits_to_f32(xb).copy()
    for l in range(first, first + n_layers):
        xn = orc.rmsnorm(h, eps)
        if l == 0:
            d = C.DEEPSEEK_V2_LITE_DENSE
            out = orc.moe_layer(oracle_desc(d), selected_host_weights(orc, d, 0, [0]), xn, threads=threads)["out"]
        else:
            r, sh = C.DEEPSEEK_V2_LITE, C.DEEPSEEK_V2_LITE_SHARED
            dr = oracle_desc(r)
            ids, _, _ = orc.route(dr, selected_host_weights(orc, r, l, []), xn)
            routed = orc.moe_layer(dr, selected_host_weights(orc, r, l, ids), xn, threads=threads)["out"]
            shared = orc.moe_layer(oracle_desc(sh), selected_host_weights(orc, sh, l, [0]), xn, threads=threads)["out"]
            out = (routed + shared).astype(np.float32)
        h = (h + out).astype(np.float32)
    return h
