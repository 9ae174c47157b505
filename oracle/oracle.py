"""ctypes bindings for the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
reference legs import this module.  The product (libumsx.so and the
unified-memory-scheduler_b200 package) never does.

`Oracle` wraps oracle/liboracle.so (the C restatement, see umsx_oracle.h for
the reference file:line each function follows).  `RefKernels` wraps
oracle/_ref/libumsx_ref.so: the reference's own tools/trace/cpu_mxfp4_vnni.cpp
and tools/trace/exact_packed_cpu.h compiled in place, used to pin the oracle.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
QUANT_Q8_0 = 8
QUANT_MXFP4 = 39
BLOCK_BYTES = {QUANT_Q8_0: 34, QUANT_MXFP4: 17}
ROUTE_TOPK_SOFTMAX, ROUTE_SOFTMAX_TOPK_NORM, ROUTE_SOFTMAX_TOPK = 0, 1, 2
ACT_SILU, ACT_SWIGLU_OAI = 0, 1

_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_u16p = C.POINTER(C.c_uint16)


def _ptr(a, t):
    if a is None:
        return C.cast(None, t)
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be contiguous"
    return a.ctypes.data_as(t)


class OrcDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "intermediate", "experts", "top_k", "quant", "routing",
                                      "activation", "fused_gate_up", "has_bias")] + \
               [(n, C.c_float) for n in ("swiglu_alpha", "swiglu_limit", "routed_scale")]


class OrcWeights(C.Structure):
    _fields_ = [("router_w", _f32p), ("router_b", _f32p), ("gate_up", _u8p), ("gate", _u8p), ("up", _u8p),
                ("down", _u8p), ("gate_up_bias", _u16p), ("down_bias", _u16p)]


@dataclass
class LayerWeights:
    """Host copies of one MoE layer in ggml layouts (what a GGUF holds)."""
    router_w: np.ndarray            # f32 [E, H]
    router_b: np.ndarray | None     # f32 [E]
    gate_up: np.ndarray | None      # u8 [E, 2I, H/32*bb]  (fused, gate rows first)
    gate: np.ndarray | None         # u8 [E, I, H/32*bb]
    up: np.ndarray | None
    down: np.ndarray                # u8 [E, H, I/32*bb]
    gate_up_bias: np.ndarray | None  # bf16 bits u16 [E, 2I]
    down_bias: np.ndarray | None     # bf16 bits u16 [E, H]


def _load(path):
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built; run `make -C oracle` (or __graft_entry__.build())")
    return C.CDLL(path)


class Oracle:
    def __init__(self, path: str | None = None):
        L = self.lib = _load(path or os.path.join(HERE, "liboracle.so"))
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_f32_to_bf16.argtypes = [C.c_float]
        L.orc_exp.restype = C.c_float
        L.orc_exp.argtypes = [C.c_float]
        L.orc_swiglu_oai.restype = C.c_float
        L.orc_swiglu_oai.argtypes = [C.c_float] * 4
        L.orc_silu_mul.restype = C.c_float
        L.orc_silu_mul.argtypes = [C.c_float] * 2
        L.orc_e8m0_half.restype = C.c_float
        L.orc_e8m0_half.argtypes = [C.c_uint8]
        L.orc_quantize_q8_0.argtypes = [_f32p, _u8p, C.c_int]
        L.orc_dot_mxfp4_q8_0.restype = C.c_float
        L.orc_dot_mxfp4_q8_0.argtypes = [C.c_int, _u8p, _u8p]
        L.orc_dot_q8_0_q8_0.restype = C.c_float
        L.orc_dot_q8_0_q8_0.argtypes = [C.c_int, _u8p, _u8p]
        L.orc_dequant_mxfp4.argtypes = [_u8p, _f32p, C.c_int64]
        L.orc_dequant_q8_0.argtypes = [_u8p, _f32p, C.c_int64]
        L.orc_gemv.argtypes = [C.c_int, C.c_int, C.c_int, _u8p, _u8p, _f32p, C.c_int]
        L.orc_logit.restype = C.c_float
        L.orc_logit.argtypes = [_f32p, _f32p, C.c_int]
        L.orc_route.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _f32p, _f32p, _f32p, C.c_int,
                                _i32p, _f32p, _f32p]
        L.orc_moe_layer.restype = C.c_int
        L.orc_moe_layer.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int, _f32p, _i32p,
                                    _f32p, _i32p, _u8p, _f32p, C.c_int]
        L.orc_moe_experts.restype = C.c_int
        L.orc_moe_experts.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights), _f32p, C.c_int, _i32p, _f32p,
                                      _f32p, _u8p, _f32p, C.c_int]
        L.orc_rmsnorm.argtypes = [_f32p, _f32p, C.c_int, C.c_float]
        L.orc_rng.restype = C.c_uint64
        L.orc_rng.argtypes = [C.c_uint64] * 3
        L.orc_gen_mxfp4.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_int, C.c_int, _u8p]
        L.orc_gen_q8_0.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, _u8p]
        L.orc_gen_normal_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, _f32p]
        L.orc_gen_normal_bf16.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, _u16p]
        L.orc_normal_scale.restype = C.c_float
        L.orc_normal_scale.argtypes = [C.c_double]

    # -- primitives --------------------------------------------------------
    def quantize_q8_0(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.shape[-1]
        rows = x.size // n
        out = np.empty((rows, n // 32 * 34), np.uint8)
        for r in range(rows):
            self.lib.orc_quantize_q8_0(_ptr(x.reshape(rows, n)[r], _f32p), _ptr(out[r], _u8p), n)
        return out.reshape(*x.shape[:-1], n // 32 * 34)

    def dot(self, quant: int, n: int, w: np.ndarray, a: np.ndarray) -> float:
        fn = self.lib.orc_dot_mxfp4_q8_0 if quant == QUANT_MXFP4 else self.lib.orc_dot_q8_0_q8_0
        return fn(n, _ptr(np.ascontiguousarray(w), _u8p), _ptr(np.ascontiguousarray(a), _u8p))

    def gemv(self, quant: int, n: int, W: np.ndarray, a: np.ndarray, threads: int = 1) -> np.ndarray:
        W = np.ascontiguousarray(W)
        rows = W.size // (n // 32 * BLOCK_BYTES[quant])
        out = np.empty(rows, np.float32)
        self.lib.orc_gemv(quant, n, rows, _ptr(W, _u8p), _ptr(np.ascontiguousarray(a), _u8p), _ptr(out, _f32p),
                          threads)
        return out

    def dequant(self, quant: int, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        fn = self.lib.orc_dequant_mxfp4 if quant == QUANT_MXFP4 else self.lib.orc_dequant_q8_0
        fn(_ptr(np.ascontiguousarray(blocks), _u8p), _ptr(out, _f32p), n)
        return out

    def exp(self, x: float) -> float:
        return self.lib.orc_exp(x)

    def rmsnorm(self, x: np.ndarray, eps: float = 1e-5) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        n = x.shape[-1]
        for r in range(x.size // n):
            self.lib.orc_rmsnorm(_ptr(x.reshape(-1, n)[r], _f32p), _ptr(out.reshape(-1, n)[r], _f32p), n, eps)
        return out

    # -- router / layer ------------------------------------------------------
    def route(self, desc: OrcDesc, w: LayerWeights, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        ids = np.empty((T, desc.top_k), np.int32)
        wt = np.empty((T, desc.top_k), np.float32)
        logits = np.empty((T, desc.experts), np.float32)
        self.lib.orc_route(desc.routing, desc.experts, desc.top_k, desc.hidden, desc.routed_scale,
                           _ptr(w.router_w, _f32p), _ptr(w.router_b, _f32p), _ptr(x, _f32p), T,
                           _ptr(ids, _i32p), _ptr(wt, _f32p), _ptr(logits, _f32p))
        return ids, wt, logits

    @staticmethod
    def _weights_struct(w: LayerWeights) -> OrcWeights:
        return OrcWeights(_ptr(w.router_w, _f32p), _ptr(w.router_b, _f32p), _ptr(w.gate_up, _u8p),
                          _ptr(w.gate, _u8p), _ptr(w.up, _u8p), _ptr(w.down, _u8p), _ptr(w.gate_up_bias, _u16p),
                          _ptr(w.down_bias, _u16p))

    def moe_layer(self, desc: OrcDesc, w: LayerWeights, x: np.ndarray, threads: int = 8):
        x = np.ascontiguousarray(x, np.float32)
        T, H, K = x.shape[0], desc.hidden, desc.top_k
        out = np.empty((T, H), np.float32)
        ids = np.empty((T, K), np.int32)
        wt = np.empty((T, K), np.float32)
        counts = np.empty(desc.experts, np.int32)
        aq = np.empty((T * K, desc.intermediate // 32 * 34), np.uint8)
        y = np.empty((T * K, H), np.float32)
        ws = self._weights_struct(w)
        rc = self.lib.orc_moe_layer(C.byref(desc), C.byref(ws), _ptr(x, _f32p), T, _ptr(out, _f32p),
                                    _ptr(ids, _i32p), _ptr(wt, _f32p), _ptr(counts, _i32p), _ptr(aq, _u8p),
                                    _ptr(y, _f32p), threads)
        if rc:
            raise ValueError("oracle rejected the layer shape")
        return dict(out=out, ids=ids, weights=wt, counts=counts, act_q8=aq, y=y)

    def moe_experts(self, desc: OrcDesc, w: LayerWeights, x: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                    threads: int = 8):
        x = np.ascontiguousarray(x, np.float32)
        T, H = x.shape[0], desc.hidden
        out = np.empty((T, H), np.float32)
        y = np.empty((ids.size, H), np.float32)
        ws = self._weights_struct(w)
        rc = self.lib.orc_moe_experts(C.byref(desc), C.byref(ws), _ptr(x, _f32p), T,
                                      _ptr(np.ascontiguousarray(ids, np.int32), _i32p),
                                      _ptr(np.ascontiguousarray(weights, np.float32), _f32p), _ptr(out, _f32p),
                                      C.cast(None, _u8p), _ptr(y, _f32p), threads)
        if rc:
            raise ValueError("oracle rejected the layer shape")
        return out, y

    # -- generator -------------------------------------------------------------
    def gen_mxfp4(self, seed, stream, first, nblocks, e_lo=119, e_span=5):
        out = np.empty(nblocks * 17, np.uint8)
        self.lib.orc_gen_mxfp4(seed, stream, first, nblocks, e_lo, e_span, _ptr(out, _u8p))
        return out

    def gen_blocks_into(self, quant, out, seed, stream, first, nblocks, threads=1):
        """Fills the uint8 array `out` (nblocks ggml blocks, C-contiguous) with the generator's blocks
        first..first+nblocks-1, split over `threads` host threads (the C generator releases the GIL)."""
        from concurrent.futures import ThreadPoolExecutor
        bb = BLOCK_BYTES[quant]
        flat = out.reshape(-1)
        assert flat.size == nblocks * bb and flat.flags["C_CONTIGUOUS"]
        per = max(1, (nblocks + threads - 1) // threads)

        def run(i):
            lo, hi = i * per, min(nblocks, (i + 1) * per)
            if lo >= hi:
                return
            ptr = flat[lo * bb:].ctypes.data_as(_u8p)
            if quant == QUANT_MXFP4:
                self.lib.orc_gen_mxfp4(seed, stream, first + lo, hi - lo, 119, 5, ptr)
            else:
                self.lib.orc_gen_q8_0(seed, stream, first + lo, hi - lo, ptr)

        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(run, range(threads)))
        return out

    def gen_q8_0(self, seed, stream, first, nblocks):
        out = np.empty(nblocks * 34, np.uint8)
        self.lib.orc_gen_q8_0(seed, stream, first, nblocks, _ptr(out, _u8p))
        return out

    def gen_normal_f32(self, seed, stream, first, n, sigma):
        out = np.empty(n, np.float32)
        self.lib.orc_gen_normal_f32(seed, stream, first, n, self.lib.orc_normal_scale(sigma), _ptr(out, _f32p))
        return out

    def gen_normal_bf16(self, seed, stream, first, n, sigma):
        out = np.empty(n, np.uint16)
        self.lib.orc_gen_normal_bf16(seed, stream, first, n, self.lib.orc_normal_scale(sigma), _ptr(out, _u16p))
        return out


class RefKernels:
    """The reference's own CPU kernels, compiled in place (oracle/_ref)."""

    def __init__(self, path: str | None = None):
        L = self.lib = _load(path or os.path.join(HERE, "_ref", "libumsx_ref.so"))
        L.ref_cpu_supported.restype = C.c_int
        L.ref_vec_dot_mxfp4_q8_0.argtypes = [C.c_int, _f32p, _u8p, _u8p]
        L.ref_pack_mxfp4x8.argtypes = [_u8p, C.c_int, C.c_int, _u8p]
        L.ref_packed_gemv.restype = C.c_int
        L.ref_packed_gemv.argtypes = [C.c_int, _f32p, _u8p, _u8p, C.c_int]
        L.ref_pack_activation.restype = C.c_int
        L.ref_pack_activation.argtypes = [_f32p, _u8p, C.c_int64]
        L.ref_packed_gemm.restype = C.c_int
        L.ref_packed_gemm.argtypes = [C.c_int, _f32p, C.c_size_t, _u8p, _u8p, C.c_int, C.c_int]
        L.ref_layer_create.restype = C.c_void_p
        L.ref_layer_create.argtypes = [C.POINTER(OrcDesc), C.POINTER(OrcWeights)]
        L.ref_layer_destroy.argtypes = [C.c_void_p]
        L.ref_layer_forward.restype = C.c_int
        L.ref_layer_forward.argtypes = [C.c_void_p, _f32p, C.c_int, _f32p, C.c_int]

    def supported(self) -> bool:
        return bool(self.lib.ref_cpu_supported())

    def vec_dot(self, n, w, a) -> float:
        out = np.zeros(1, np.float32)
        self.lib.ref_vec_dot_mxfp4_q8_0(n, _ptr(out, _f32p), _ptr(np.ascontiguousarray(w), _u8p),
                                        _ptr(np.ascontiguousarray(a), _u8p))
        return float(out[0])

    def pack(self, raw: np.ndarray, n: int, rows: int) -> np.ndarray:
        out = np.empty(rows // 8 * (n // 32) * 136, np.uint8)
        self.lib.ref_pack_mxfp4x8(_ptr(np.ascontiguousarray(raw), _u8p), n, rows, _ptr(out, _u8p))
        return out

    def gemv(self, n, packed, a, columns) -> np.ndarray:
        out = np.empty(columns, np.float32)
        if self.lib.ref_packed_gemv(n, _ptr(out, _f32p), _ptr(packed, _u8p), _ptr(np.ascontiguousarray(a), _u8p),
                                    columns):
            raise ValueError("reference packed GEMV rejected the shape")
        return out

    def pack_activation(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        k = x.shape[-1]
        out = np.empty(k // 32 * 136, np.uint8)
        if self.lib.ref_pack_activation(_ptr(x, _f32p), _ptr(out, _u8p), k):
            raise ValueError("reference activation packing rejected the shape")
        return out

    def gemm(self, n, packed_w, packed_a, rows, columns, stride, fill=-123.25) -> np.ndarray:
        out = np.full(rows * stride, fill, np.float32)
        if self.lib.ref_packed_gemm(n, _ptr(out, _f32p), stride, _ptr(packed_w, _u8p), _ptr(packed_a, _u8p), rows,
                                    columns):
            raise ValueError("reference packed GEMM rejected the shape")
        return out

    def layer(self, desc: OrcDesc, w: LayerWeights):
        ws = Oracle._weights_struct(w)
        h = self.lib.ref_layer_create(C.byref(desc), C.byref(ws))
        if not h:
            raise ValueError("reference layer driver supports fused MXFP4 layers only")
        return h

    def layer_forward(self, handle, x: np.ndarray, hidden: int, threads: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty((x.shape[0], hidden), np.float32)
        self.lib.ref_layer_forward(handle, _ptr(x, _f32p), x.shape[0], _ptr(out, _f32p), threads)
        return out

    def layer_destroy(self, handle):
        self.lib.ref_layer_destroy(handle)
