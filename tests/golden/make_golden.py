#!/usr/bin/env python3
"""Regenerate the golden vectors in tests/golden/ from the REFERENCE's own CPU kernels.

Runs only where the reference tree is present (it needs oracle/_ref/libumsx_ref.so,
built by `make -C oracle ref` from tools/trace/cpu_mxfp4_vnni.cpp and
tools/trace/exact_packed_cpu.h).  The outputs are small .npz files that travel with
the repository; the tests check the C oracle and the CUDA kernels against them
without the reference tree.

Fixtures (each mirrors a reference test, path inside the reference project):
  exact_packed_417.npz  tests/test_exact_packed_cpu.cpp:53-145 -- the same std::mt19937(417)
                        stream (replayed with numpy's legacy MT19937, which is bit-identical),
                        n in {64,256,2880}, columns in {8,16,64}, rows in {4,8}, E8M0 96..135
                        with e=0/e=1 forced, a -128 activation code, stride canary -123.25,
                        and the 2880x2880 timing GEMV (E8M0 120..127).
  compatible_down.npz   tools/trace/hybrid_layer.cpp:964-979 adversarial MXFP4 down bank
                        (all 16 codes, E8M0 {0,1,2,120,126,127,128,130}) x activation patterns
                        sine / zero / q8-ties of :593-607 and :1058-1066, 7 rows x 4 ranks
                        (tests/test_compatible_down.py:13-48).
  quantized_down.npz    tests/test_quantized_cuda.cpp:31-41: jobs {(0,0,0),(1,0,2),(0,1,0)},
                        12 samples (zero input, sin pattern, 0x80 in every Q8 block at sample 11).

Expected outputs come from the reference's ggml_vec_dot_mxfp4_q8_0 and exact packed
GEMV/GEMM; the Q8_0 activations come from the oracle's quantizer (ggml's own
quantize_row_q8_0 is not in the reference tree).
"""
import ctypes
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle.oracle import Oracle, RefKernels  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
libm = ctypes.CDLL("libm.so.6")
libm.sinf.restype = ctypes.c_float
libm.sinf.argtypes = [ctypes.c_float]


class MT19937:
    """std::mt19937 replay (numpy's legacy seeding is init_genrand)."""

    def __init__(self, seed):
        self.bg = np.random.RandomState(seed)._bit_generator

    def raw(self, n=1):
        return self.bg.random_raw(n).astype(np.uint64)

    def uniform(self, n, lo, hi):
        # libstdc++ generate_canonical<float,24> with one 32-bit draw, then a + u*(b-a)
        f = (self.raw(n).astype(np.float32) / np.float32(4294967296.0)).astype(np.float32)
        f = np.where(f >= 1, np.nextafter(np.float32(1), np.float32(0)), f).astype(np.float32)
        return (f * np.float32(hi - lo) + np.float32(lo)).astype(np.float32)


def exact_packed_inputs():
    """Yields the reference test's (n, columns, weights, floats) in draw order."""
    g = MT19937(417)
    for n in (64, 256, 2880):
        blocks = n // 32
        for columns in (8, 16, 64):
            w = np.empty((columns * blocks, 17), np.uint8)
            for b in range(columns * blocks):
                w[b, 0] = 96 + int(g.raw()[0] % 40)
                w[b, 1:] = (g.raw(16) & 0xFF).astype(np.uint8)
            w[0, 0] = 0
            w[1, 0] = 1
            floats = g.uniform(n * 8, -8, 8)
            yield n, columns, w, floats
    n = columns = 2880
    blocks = n // 32
    w = np.empty((columns * blocks, 17), np.uint8)
    for b in range(columns * blocks):
        w[b, 0] = 120 + int(g.raw()[0] % 8)
        w[b, 1:] = (g.raw(16) & 0xFF).astype(np.uint8)
    x = g.uniform(n, -8, 8)
    yield n, -columns, w, x


def make_exact_packed(orc, ref):
    out, h = {}, hashlib.sha256()
    for n, columns, w, floats in exact_packed_inputs():
        h.update(w.tobytes())
        h.update(floats.tobytes())
        blocks = n // 32
        if columns < 0:  # the timing GEMV
            columns = -columns
            a = orc.quantize_q8_0(floats)
            packed = ref.pack(w, n, columns)
            got = ref.gemv(n, packed, a, columns)
            out["timing_gemv_2880"] = got
            continue
        act = orc.quantize_q8_0(floats.reshape(8, n))  # [8, blocks*34]
        act_flat = act.reshape(-1).copy()
        act_flat[2] = 0x80  # activations[0].qs[0] = -128
        native = np.array([ref.vec_dot(n, w[c * blocks:(c + 1) * blocks], act_flat[:blocks * 34])
                           for c in range(columns)], np.float32)
        packed = ref.pack(w, n, columns)
        gemv = ref.gemv(n, packed, act_flat[:blocks * 34], columns)
        assert native.tobytes() == gemv.tobytes(), "reference packed GEMV disagrees with reference vec_dot"
        out[f"gemv_{n}_{columns}"] = gemv
        for rows in (4, 8):
            stride = columns + 3
            pa = np.concatenate([ref.pack_activation(floats[g4 * 4 * n:(g4 + 1) * 4 * n].reshape(4, n))
                                 for g4 in range(rows // 4)])
            gemm = ref.gemm(n, packed, pa, rows, columns, stride)
            expected = np.full(rows * stride, -123.25, np.float32)
            for r in range(rows):
                for c in range(columns):
                    expected[r * stride + c] = ref.vec_dot(n, w[c * blocks:(c + 1) * blocks], act[r])
            assert expected.tobytes() == gemm.tobytes(), "reference packed GEMM disagrees with reference vec_dot"
            out[f"gemm_{n}_{columns}_{rows}"] = gemm
    out["inputs_sha256"] = np.frombuffer(h.digest(), np.uint8)
    np.savez_compressed(os.path.join(OUT, "exact_packed_417.npz"), **out)


def compatible_weights(experts=4, hidden=64, intermediate=128):
    exps = [0, 1, 2, 120, 126, 127, 128, 130]
    nb = intermediate // 32
    w = np.empty((experts * hidden * nb, 17), np.uint8)
    for b in range(w.shape[0]):
        w[b, 0] = exps[(b // nb) % 8]
        for j in range(16):
            w[b, 1 + j] = ((b + j) % 16) | ((((b * 7 + j * 3) % 16)) << 4)
    return w


def activation_input(size, sample, pattern, self_test=True):
    mag = (0.2 if sample % 3 == 0 else 50.0 if sample % 3 == 1 else 500.0) if self_test else 0.2
    v = np.empty(size, np.float32)
    for i in range(size):
        if pattern == "zero":
            v[i] = 0.0
        elif pattern == "q8-ties":
            v[i] = 127.0 if i % 32 == 0 else -127.0 if i % 32 == 1 else \
                np.float32(-1.0 if i % 2 else 1.0) * np.float32(0.5 + float((i + 7 * sample) % 31))
        else:
            arg = np.float32(np.float32((i + 1) * (sample + 3)) * np.float32(0.017))
            v[i] = np.float32(mag) * np.float32(libm.sinf(float(arg)))
    return v


def make_compatible(orc, ref):
    w = compatible_weights()
    hidden, inter, nb, rows, active = 64, 128, 4, 7, 4
    out = {"weights": w}
    for pattern in ("sine", "zero", "q8-ties"):
        for sample in range(3):
            v = activation_input(inter * active * rows, sample, pattern)
            if pattern == "sine":
                mags = np.array([1.0, 0.001, 0.00000001, 16384.0], np.float32)
                for i in range(v.size):
                    v[i] = np.float32(v[i] * mags[(i // 32 + sample) % 4])
            act = orc.quantize_q8_0(v.reshape(rows * active, inter))
            res = np.empty((rows * active, hidden), np.float32)
            for j in range(rows * active):
                e = j % active
                for h in range(hidden):
                    row = w[(e * hidden + h) * nb:(e * hidden + h + 1) * nb]
                    res[j, h] = ref.vec_dot(inter, row, act[j])
            out[f"{pattern}_{sample}_act"] = act
            out[f"{pattern}_{sample}_out"] = res
    np.savez_compressed(os.path.join(OUT, "compatible_down.npz"), **out)


def make_quantized_down(orc, ref):
    hidden, inter, experts = 64, 128, 3
    nb = inter // 32
    w = orc.gen_mxfp4(4170, 1, 0, experts * hidden * nb).reshape(experts * hidden * nb, 17)
    jobs = np.array([[0, 0, 0], [1, 0, 2], [0, 1, 0]], np.int64)  # (row, rank, expert)
    out = {"weights": w, "jobs": jobs}
    for sample in range(12):
        v = np.empty(len(jobs) * inter, np.float32)
        for i in range(v.size):
            v[i] = 0.0 if sample == 0 else np.float32(
                libm.sinf(float(np.float32(np.float32(i * 13 + sample * 31) * np.float32(0.07))))) * np.float32(sample)
        act = orc.quantize_q8_0(v.reshape(len(jobs), inter))
        if sample == 11:
            flat = act.reshape(-1)
            flat[2::34] = 0x80
        res = np.empty((len(jobs), hidden), np.float32)
        for j, (_, _, e) in enumerate(jobs):
            for h in range(hidden):
                res[j, h] = ref.vec_dot(inter, w[(e * hidden + h) * nb:(e * hidden + h + 1) * nb], act[j])
        out[f"s{sample}_act"] = act
        out[f"s{sample}_out"] = res
    np.savez_compressed(os.path.join(OUT, "quantized_down.npz"), **out)


def main():
    orc, ref = Oracle(), RefKernels()
    if not ref.supported():
        sys.exit("the reference kernels need AVX-512 VNNI/BW/VL and F16C on this host")
    make_exact_packed(orc, ref)
    make_compatible(orc, ref)
    make_quantized_down(orc, ref)
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)), "bytes")


if __name__ == "__main__":
    main()
