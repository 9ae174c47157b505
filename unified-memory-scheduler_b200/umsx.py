"""Python bindings over libumsx's C ABI (include/umsx.h).

Mirrors the reference's expert interfaces (paths inside appatalks/unified-memory-scheduler):
  MoeLayer.forward        build_moe_ffn expert branch + rank-order sum
                          (third_party/patches/llama-b11669-hybrid-experts.patch:1394-1683, :1911-1916)
  MoeLayer.route          router + top-k with lower-index ties (tools/trace/topk-tie-probe.cpp:111-113)
  MoeLayer.expert_down_q8 Mxfp4NativeCudaDown::execute (tools/engine/quantized_cuda.cu:413-453)
  MoeLayer.mul_mat_id     ggml MUL_MAT_ID with -1 masked ids (hybrid patch :617-621)
  combine                 ExpertPlan::execute's rank-order combine (tools/engine/expert_dispatch.cpp:77-87)
Errors raise UmsxError carrying the C status, as the reference raises
std::invalid_argument / std::runtime_error.  Device buffers are torch CUDA
tensors (plumbing only); there is no CPU fallback: without libumsx.so or a GPU
every call fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libumsx.so")

OK, EINVAL, ENOTRESIDENT, EOOM, ETIMEOUT, EDEVICE, EUNSUPPORTED, ENONFINITE = range(8)
STATUS_NAMES = ["OK", "EINVAL", "ENOTRESIDENT", "EOOM", "ETIMEOUT", "EDEVICE", "EUNSUPPORTED", "ENONFINITE"]
QUANT_Q8_0, QUANT_MXFP4 = 8, 39
ROUTE_TOPK_SOFTMAX, ROUTE_SOFTMAX_TOPK_NORM, ROUTE_SOFTMAX_TOPK = 0, 1, 2
ACT_SILU, ACT_SWIGLU_OAI = 0, 1
DTYPE_F32, DTYPE_BF16 = 0, 1
BANK_LFU, BANK_LRU = 0, 1
BANK_STAT_NAMES = ("dispatches", "demands", "hits", "misses", "admissions", "evictions", "transient", "halvings",
                   "upload_bytes")
PROJ_GATE_UP, PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2, 3
BLOCK_BYTES = {QUANT_Q8_0: 34, QUANT_MXFP4: 17}

# exported symbols of include/umsx.h (the tests check each one is present)
EXPORTS = ["umsx_moe_create", "umsx_moe_create_synthetic", "umsx_moe_destroy", "umsx_moe_set_router", "umsx_moe_forward",
           "umsx_moe_create_banked", "umsx_moe_bank_stats", "umsx_bank_simulate",
           "umsx_moe_forward_host", "umsx_moe_forward_jobs", "umsx_moe_status", "umsx_route", "umsx_expert_down_q8", "umsx_mul_mat_id",
           "umsx_combine",
           "umsx_moe_export_expert", "umsx_stack_create", "umsx_stack_create_mixed", "umsx_stack_destroy", "umsx_stack_forward",
           "umsx_stack_forward_host", "umsx_stack_status", "umsx_stack_set_timing", "umsx_stack_stage_times", "umsx_stack_inject_fault",
           "umsx_route_static", "umsx_ep_create", "umsx_ep_handle", "umsx_ep_connect", "umsx_ep_set_wait",
           "umsx_ep_destroy", "umsx_ep_stack_create", "umsx_ep_stack_destroy", "umsx_ep_stack_forward",
           "umsx_ep_stack_forward_host", "umsx_ep_stack_status", "umsx_ep_prefill_create", "umsx_ep_prefill_handle",
           "umsx_ep_prefill_connect", "umsx_ep_prefill_forward", "umsx_ep_prefill_forward_host", "umsx_ep_prefill_loads",
           "umsx_ep_prefill_status", "umsx_ep_prefill_destroy",
           "umsx_gguf_load_experts", "umsx_gguf_experts_free", "umsx_moe_create_gguf",
           "umsx_kernel_launches", "umsx_last_error", "umsx_version"]


class UmsxError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"umsx {name}: {message}")


class Desc(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "intermediate", "experts", "top_k", "quant", "routing", "activation",
                                        "fused_gate_up", "has_bias", "has_router_bias")] + \
               [(n, C.c_float) for n in ("swiglu_alpha", "swiglu_limit", "routed_scale")] + \
               [(n, C.c_int32) for n in ("max_tokens", "ep_rank", "ep_world")]


class Weights(C.Structure):
    _fields_ = [("router_w", C.c_void_p), ("router_b", C.c_void_p), ("gate_up", C.c_void_p), ("gate", C.c_void_p),
                ("up", C.c_void_p), ("down", C.c_void_p), ("gate_up_bias", C.c_void_p), ("down_bias", C.c_void_p)]


class GgufExpertsC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "intermediate", "experts", "n_ids")] + \
               [("quant", C.c_int32 * 3), ("stride", C.c_uint64 * 3), ("packed", C.c_void_p * 3),
                ("values", C.c_void_p * 3), ("bias", C.c_void_p * 3), ("owner", C.c_void_p)]


_lib = None


def lib():
    """Loads libumsx.so (built in-tree by __graft_entry__.build()); raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
    L = C.CDLL(LIB_PATH)
    vp, i32, sz, u64 = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64
    sig = {
        "umsx_moe_create": (i32, [C.POINTER(Desc), C.POINTER(Weights), i32, sz, C.POINTER(vp)]),
        "umsx_moe_create_synthetic": (i32, [C.POINTER(Desc), u64, C.c_uint32, C.c_float, C.c_float, C.c_float, i32, sz,
                                            C.POINTER(vp)]),
        "umsx_moe_destroy": (None, [vp]),
        "umsx_moe_create_banked": (i32, [C.POINTER(Desc), C.POINTER(Weights), i32, i32, i32, sz, C.POINTER(vp)]),
        "umsx_moe_bank_stats": (i32, [vp, vp, i32, vp, i32]),
        "umsx_bank_simulate": (i32, [i32, i32, i32, i32, vp, vp, vp, vp]),
        "umsx_moe_set_router": (i32, [vp, vp, vp]),
        "umsx_moe_forward": (i32, [vp, vp, i32, i32, vp, vp, vp, vp]),
        "umsx_moe_forward_host": (i32, [vp, vp, i32, i32, vp, vp]),
        "umsx_moe_forward_jobs": (i32, [vp, vp, i32, i32, vp, vp, vp, vp]),
        "umsx_moe_status": (i32, [vp, vp]),
        "umsx_stack_status": (i32, [vp, vp]),
        "umsx_route": (i32, [vp, vp, i32, i32, vp, vp, vp, vp]),
        "umsx_expert_down_q8": (i32, [vp, vp, vp, i32, vp, vp]),
        "umsx_mul_mat_id": (i32, [vp, i32, vp, i32, vp, i32, i32, vp, vp]),
        "umsx_combine": (i32, [vp, vp, i32, i32, i32, vp, vp]),
        "umsx_moe_export_expert": (i32, [vp, i32, i32, vp, sz]),
        "umsx_stack_create": (i32, [C.POINTER(vp), i32, i32, C.c_float, C.POINTER(vp)]),
        "umsx_stack_create_mixed": (i32, [C.POINTER(vp), C.POINTER(vp), i32, i32, C.c_float, C.POINTER(vp)]),
        "umsx_stack_destroy": (None, [vp]),
        "umsx_stack_forward": (i32, [vp, vp, i32, i32, vp, vp]),
        "umsx_stack_forward_host": (i32, [vp, vp, i32, i32, vp, vp]),
        "umsx_stack_set_timing": (i32, [vp, i32]),
        "umsx_stack_stage_times": (i32, [vp, C.POINTER(C.c_float), i32]),
        "umsx_stack_inject_fault": (i32, [vp, i32, C.c_int64]),
        "umsx_route_static": (i32, [vp, i32, i32, vp, vp, i32, i32, i32, i32, C.c_float, vp, vp, vp, vp]),
        "umsx_ep_create": (i32, [i32, i32, i32, i32, i32, C.POINTER(vp)]),
        "umsx_ep_handle": (i32, [vp, vp, sz]),
        "umsx_ep_connect": (i32, [vp, vp, sz]),
        "umsx_ep_set_wait": (i32, [vp, C.c_int64]),
        "umsx_ep_destroy": (None, [vp]),
        "umsx_ep_stack_create": (i32, [vp, C.POINTER(vp), i32, C.c_float, C.POINTER(vp)]),
        "umsx_ep_stack_destroy": (None, [vp]),
        "umsx_ep_stack_forward": (i32, [vp, vp, i32, vp, vp]),
        "umsx_ep_stack_forward_host": (i32, [vp, vp, i32, vp, vp]),
        "umsx_ep_stack_status": (i32, [vp, vp]),
        "umsx_ep_prefill_create": (i32, [vp, C.POINTER(vp), i32, i32, C.c_float, C.POINTER(vp)]),
        "umsx_ep_prefill_handle": (i32, [vp, vp, sz]),
        "umsx_ep_prefill_connect": (i32, [vp, vp, sz]),
        "umsx_ep_prefill_forward": (i32, [vp, vp, i32, i32, vp, vp]),
        "umsx_ep_prefill_forward_host": (i32, [vp, vp, i32, i32, vp, vp]),
        "umsx_ep_prefill_loads": (i32, [vp, vp, i32]),
        "umsx_ep_prefill_status": (i32, [vp, vp]),
        "umsx_ep_prefill_destroy": (None, [vp]),
        "umsx_gguf_load_experts": (i32, [C.c_char_p, i32, vp, i32, i32, C.POINTER(GgufExpertsC)]),
        "umsx_gguf_experts_free": (None, [C.POINTER(GgufExpertsC)]),
        "umsx_moe_create_gguf": (i32, [C.POINTER(Desc), C.c_char_p, i32, i32, sz, C.POINTER(vp)]),
        "umsx_kernel_launches": (u64, []),
        "umsx_last_error": (C.c_char_p, []),
        "umsx_version": (i32, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int):
    if status != OK:
        raise UmsxError(status, lib().umsx_last_error().decode())


def kernel_launches() -> int:
    return int(lib().umsx_kernel_launches())


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _np_ptr(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _stream(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return C.c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)


def _dtype_code(t):
    import torch
    if t.dtype == torch.float32:
        return DTYPE_F32
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    raise UmsxError(EINVAL, f"x must be float32 or bfloat16, got {t.dtype}")


def bank_simulate(experts: int, slots: int, policy: int, dispatches):
    """Runs the bank policy alone on the host (umsx_bank_simulate).  `dispatches` is a list of
    (expert list, admit) pairs: admit=True for a one-token dispatch (its top-k in rank order),
    False for a batch's distinct experts (lookup).  Returns (slots per dispatch, stats dict)."""
    import numpy as np
    counts = np.array([len(sel) if admit else -len(sel) for sel, admit in dispatches], dtype=np.int32)
    flat = np.array([e for sel, _ in dispatches for e in sel], dtype=np.int32)
    out = np.full(len(flat), -2, dtype=np.int32)
    st = np.zeros(len(BANK_STAT_NAMES), dtype=np.uint64)
    check(lib().umsx_bank_simulate(experts, slots, policy, len(dispatches), _np_ptr(counts), _np_ptr(flat),
                                   _np_ptr(out), _np_ptr(st)))
    res, at = [], 0
    for sel, _ in dispatches:
        res.append(out[at:at + len(sel)].tolist())
        at += len(sel)
    return res, {k: int(v) for k, v in zip(BANK_STAT_NAMES, st)}


def combine(y, weights, out=None, stream=None):
    """out[t] = sum_r w[t,r] * y[t,r] in rank order (y: [T,K,W] f32 CUDA, weights [T,K])."""
    import torch
    T, K, W = y.shape
    out = out if out is not None else torch.empty((T, W), dtype=torch.float32, device=y.device)
    check(lib().umsx_combine(_ptr(y), _ptr(weights), T, K, W, _ptr(out), _stream(stream)))
    return out


def route_static(x, router_w, router_b, experts: int, top_k: int, routing: int, routed_scale: float = 1.0,
                 stream=None):
    """umsx_route_static: routing without a layer handle, using only the library's fixed scratch.

    For callers that may not allocate device memory.  The output tensors here are
    allocated by torch for convenience; the C entry point itself allocates nothing.
    Calls that overlap on the GPU share the scratch and race."""
    import torch
    T, H = x.shape
    ids = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    counts = torch.empty(experts, dtype=torch.int32, device=x.device)
    check(lib().umsx_route_static(_ptr(x), _dtype_code(x), T, _ptr(router_w), _ptr(router_b), H, experts, top_k,
                                  routing, routed_scale, _ptr(ids), _ptr(w), _ptr(counts), _stream(stream)))
    return ids, w, counts


def load_gguf_experts(first_shard: str, layer: int, ids, dequantize: bool = True) -> dict:
    """The selected experts of one layer from a GGUF checkpoint (the reference's load_gguf_experts,
    tools/engine/gguf_experts.cpp:45-140): per projection ("gate", "up", "down") the ggml type, the
    raw block bytes [n_ids][stride] (uint8), the fp32 values [n_ids][rows][cols] when dequantize,
    and the fp32 bias [n_ids][len] when the file has one.  Raises UmsxError (EINVAL) on the
    reference's validation failures."""
    import numpy as np
    ids_np = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
    out = GgufExpertsC()
    L = lib()
    check(L.umsx_gguf_load_experts(os.fsencode(first_shard), int(layer), ids_np.ctypes.data, int(ids_np.size),
                                   int(bool(dequantize)), C.byref(out)))
    try:
        n, H, I = out.n_ids, out.hidden, out.intermediate
        res = {"hidden": H, "intermediate": I, "experts": out.experts, "ids": ids_np.copy()}
        for p, name in enumerate(("gate", "up", "down")):
            rows, cols = (I, H) if p < 2 else (H, I)
            stride = int(out.stride[p])
            d = {"type": int(out.quant[p]), "stride": stride,
                 "packed": np.ctypeslib.as_array(C.cast(out.packed[p], C.POINTER(C.c_uint8)),
                                                 shape=(n, stride)).copy()}
            if out.values[p]:
                d["values"] = np.ctypeslib.as_array(C.cast(out.values[p], C.POINTER(C.c_float)),
                                                    shape=(n, rows, cols)).copy()
            if out.bias[p]:
                d["bias"] = np.ctypeslib.as_array(C.cast(out.bias[p], C.POINTER(C.c_float)), shape=(n, rows)).copy()
            res[name] = d
        return res
    finally:
        L.umsx_gguf_experts_free(C.byref(out))


class MoeLayer:
    """One MoE layer resident on a GPU (the handle owns the repacked expert weights)."""

    def __init__(self, desc: Desc, weights: dict | None = None, *, synthetic: dict | None = None,
                 gguf: tuple | None = None, bank: tuple | None = None, device: int = 0, reserve_bytes: int = 1 << 30):
        """bank = (slots, BANK_LFU | BANK_LRU) with host `weights`: a banked layer (umsx_moe_create_banked)
        whose experts live in pinned host memory and enter `slots` device slots by the policy."""
        self.desc = desc
        self.device = device
        self._h = C.c_void_p()
        L = lib()
        if gguf is not None:  # (first shard path, layer index)
            path, layer = gguf
            check(L.umsx_moe_create_gguf(C.byref(desc), os.fsencode(path), int(layer), device, reserve_bytes,
                                         C.byref(self._h)))
        elif synthetic is not None:
            s = synthetic
            check(L.umsx_moe_create_synthetic(C.byref(desc), s["seed"], s.get("layer", 0), s.get("router_sigma", 0.02),
                                              s.get("router_bias_sigma", 0.1), s.get("bias_sigma", 0.02), device,
                                              reserve_bytes, C.byref(self._h)))
        else:
            w = weights
            self._keep = w  # host arrays must stay alive during create
            ws = Weights(*[_np_ptr(w.get(k)) for k in ("router_w", "router_b", "gate_up", "gate", "up", "down",
                                                      "gate_up_bias", "down_bias")])
            if bank is not None:
                check(L.umsx_moe_create_banked(C.byref(desc), C.byref(ws), int(bank[0]), int(bank[1]), device,
                                               reserve_bytes, C.byref(self._h)))
            else:
                check(L.umsx_moe_create(C.byref(desc), C.byref(ws), device, reserve_bytes, C.byref(self._h)))
            self._keep = None

    def close(self):
        if self._h:
            lib().umsx_moe_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x, out=None, ids=None, weights=None, stream=None):
        import torch
        T = x.shape[0]
        out = out if out is not None else torch.empty((T, self.desc.hidden), dtype=torch.float32, device=x.device)
        check(lib().umsx_moe_forward(self._h, _ptr(x), _dtype_code(x), T, _ptr(out), _ptr(ids), _ptr(weights),
                                     _stream(stream)))
        return out

    def forward_jobs(self, x, y=None, ids=None, weights=None, stream=None):
        """Expert-parallel share of the layer (umsx_moe_forward_jobs): routes all T rows, writes the
        outputs of the jobs whose expert this handle holds into y [T, k, H] f32 (other rows untouched).
        Returns (y, ids [T, k] int32, weights [T, k] f32)."""
        import torch
        T, K, H = x.shape[0], self.desc.top_k, self.desc.hidden
        y = y if y is not None else torch.zeros((T, K, H), dtype=torch.float32, device=x.device)
        ids = ids if ids is not None else torch.empty((T, K), dtype=torch.int32, device=x.device)
        weights = weights if weights is not None else torch.empty((T, K), dtype=torch.float32, device=x.device)
        check(lib().umsx_moe_forward_jobs(self._h, _ptr(x), _dtype_code(x), T, _ptr(ids), _ptr(weights), _ptr(y),
                                          _stream(stream)))
        return y, ids, weights

    def forward_host(self, x_host, out_host, stream=None):
        """x_host / out_host: pinned (or pageable) CPU torch tensors; synchronous."""
        check(lib().umsx_moe_forward_host(self._h, _ptr(x_host), _dtype_code(x_host), x_host.shape[0], _ptr(out_host),
                                          _stream(stream)))
        return out_host

    def set_router(self, router_w, router_b=None):
        """Replaces the router from host arrays (umsx_moe_set_router): router_w float32 [E, H],
        router_b float32 [E] exactly when the layer has a router bias."""
        import numpy as np
        w = np.ascontiguousarray(router_w, dtype=np.float32)
        b = None if router_b is None else np.ascontiguousarray(router_b, dtype=np.float32)
        check(lib().umsx_moe_set_router(self._h, _np_ptr(w), _np_ptr(b)))

    def bank_stats(self):
        """Counters of a banked layer (umsx_moe_bank_stats): a dict of BANK_STAT_NAMES, plus
        "slot_of_expert" (int32 [E], -1 where not resident)."""
        import numpy as np
        st = np.zeros(len(BANK_STAT_NAMES), dtype=np.uint64)
        slots = np.zeros(self.desc.experts, dtype=np.int32)
        check(lib().umsx_moe_bank_stats(self._h, _np_ptr(st), len(st), _np_ptr(slots), len(slots)))
        d = {k: int(v) for k, v in zip(BANK_STAT_NAMES, st)}
        d["slot_of_expert"] = slots
        return d

    def status(self, stream=None):
        """Raises UmsxError (ENONFINITE / ETIMEOUT) for what the handle's earlier calls on the stream
        recorded on the device; clears the record (umsx_moe_status)."""
        check(lib().umsx_moe_status(self._h, _stream(stream)))

    def route(self, x, stream=None):
        import torch
        T, K, E = x.shape[0], self.desc.top_k, self.desc.experts
        ids = torch.empty((T, K), dtype=torch.int32, device=x.device)
        w = torch.empty((T, K), dtype=torch.float32, device=x.device)
        counts = torch.empty(E // max(1, self.desc.ep_world), dtype=torch.int32, device=x.device)
        check(lib().umsx_route(self._h, _ptr(x), _dtype_code(x), T, _ptr(ids), _ptr(w), _ptr(counts), _stream(stream)))
        return ids, w, counts

    def expert_down_q8(self, packed_q8, experts, stream=None):
        """packed_q8: uint8 CUDA [jobs, I/32*34]; experts: host int32 numpy [jobs] -> [jobs, H] f32."""
        import numpy as np
        import torch
        experts = np.ascontiguousarray(experts, dtype=np.int32)
        jobs = int(experts.shape[0])
        out = torch.empty((jobs, self.desc.hidden), dtype=torch.float32, device=packed_q8.device)
        check(lib().umsx_expert_down_q8(self._h, _ptr(packed_q8), _np_ptr(experts), jobs, _ptr(out), _stream(stream)))
        return out

    def mul_mat_id(self, proj: int, b, ids, stream=None):
        """b: f32 CUDA [T, n_b, K]; ids: int32 CUDA [T, n_ids] (-1 masks) -> [T, n_ids, N] f32."""
        import torch
        T, n_b, _ = b.shape
        n_ids = ids.shape[1]
        N = {PROJ_GATE_UP: 2 * self.desc.intermediate, PROJ_GATE: self.desc.intermediate,
             PROJ_UP: self.desc.intermediate, PROJ_DOWN: self.desc.hidden}[proj]
        dst = torch.empty((T, n_ids, N), dtype=torch.float32, device=b.device)
        check(lib().umsx_mul_mat_id(self._h, proj, _ptr(b), n_b, _ptr(ids), n_ids, T, _ptr(dst), _stream(stream)))
        return dst

    def export_expert(self, proj: int, expert: int):
        import numpy as np
        d = self.desc
        rows, cols = {PROJ_GATE_UP: (2 * d.intermediate, d.hidden), PROJ_GATE: (d.intermediate, d.hidden),
                      PROJ_UP: (d.intermediate, d.hidden), PROJ_DOWN: (d.hidden, d.intermediate)}[proj]
        out = np.empty(rows * (cols // 32) * BLOCK_BYTES[d.quant], np.uint8)
        check(lib().umsx_moe_export_expert(self._h, proj, expert, _np_ptr(out), out.nbytes))
        return out


class MoeStack:
    """h <- h + MoE_l(RMSNorm(h)) over a list of MoeLayer (one CUDA graph replay per call).

    shared: optional list (one entry per layer, None for none) of one-expert top-1 MoeLayer handles
    holding each layer's shared experts; their output is the term after the routed ones in the
    layer's rank-order combine (umsx_stack_create_mixed).  With `shared`, the layers may differ in
    shape (e.g. a dense FFN as layer 0, itself a one-expert top-1 layer)."""

    STAGES = ("router", "gate_up", "down", "combine")

    def __init__(self, layers: list, max_tokens: int, rms_eps: float = 1e-5, shared: list | None = None):
        self.layers = list(layers)
        self.shared = list(shared) if shared is not None else None
        self.hidden = self.layers[0].desc.hidden
        arr = (C.c_void_p * len(self.layers))(*[l._h for l in self.layers])
        self._h = C.c_void_p()
        if self.shared is None:
            check(lib().umsx_stack_create(arr, len(self.layers), max_tokens, rms_eps, C.byref(self._h)))
        else:
            if len(self.shared) != len(self.layers):
                raise UmsxError(EINVAL, "one shared entry (or None) per layer")
            sh = (C.c_void_p * len(self.layers))(*[None if x is None else x._h for x in self.shared])
            check(lib().umsx_stack_create_mixed(arr, sh, len(self.layers), max_tokens, rms_eps, C.byref(self._h)))

    def close(self):
        if self._h:
            lib().umsx_stack_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x, out=None, stream=None):
        import torch
        out = out if out is not None else torch.empty((x.shape[0], self.hidden), dtype=torch.float32, device=x.device)
        check(lib().umsx_stack_forward(self._h, _ptr(x), _dtype_code(x), x.shape[0], _ptr(out), _stream(stream)))
        return out

    def forward_host(self, x_host, out_host, stream=None):
        check(lib().umsx_stack_forward_host(self._h, _ptr(x_host), _dtype_code(x_host), x_host.shape[0],
                                            _ptr(out_host), _stream(stream)))
        return out_host

    def status(self, stream=None):
        """umsx_stack_status: raises for a non-finite layer output or a wait that gave up."""
        check(lib().umsx_stack_status(self._h, _stream(stream)))

    def set_timing(self, enable: bool = True):
        check(lib().umsx_stack_set_timing(self._h, int(enable)))

    def inject_fault(self, cta: int = 0, wait_limit_cycles: int = 2_000_000):
        """Test hook (umsx_stack_inject_fault): the next one-launch forward loses CTA `cta`'s first
        grid-barrier arrival, its bounded waits run out and the call reports ETIMEOUT."""
        check(lib().umsx_stack_inject_fault(self._h, int(cta), int(wait_limit_cycles)))

    def stage_times(self) -> dict:
        ms = (C.c_float * 4)()
        check(lib().umsx_stack_stage_times(self._h, ms, 4))
        return dict(zip(self.STAGES, [float(v) for v in ms]))
