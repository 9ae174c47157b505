"""The C oracle against the reference's own kernels (golden vectors) -- CPU only.

The golden files were produced by tests/golden/make_golden.py from the
reference's tools/trace/cpu_mxfp4_vnni.cpp and tools/trace/exact_packed_cpu.h
compiled in place.  Here the oracle must reproduce them bit for bit.
"""
import os

import numpy as np
import pytest

from tests.golden.make_golden import activation_input, compatible_weights, exact_packed_inputs  # noqa: F401
from oracle.oracle import QUANT_MXFP4


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_exact_packed_golden(oracle, golden_dir):
    """tests/test_exact_packed_cpu.cpp:53-145: native GEMV/GEMM cases, seed 417."""
    g = np.load(os.path.join(golden_dir, "exact_packed_417.npz"))
    import hashlib
    h = hashlib.sha256()
    checks = 0
    for n, columns, w, floats in exact_packed_inputs():
        h.update(w.tobytes())
        h.update(floats.tobytes())
        blocks = n // 32
        if columns < 0:
            columns = -columns
            a = oracle.quantize_q8_0(floats)
            got = oracle.gemv(QUANT_MXFP4, n, w, a, threads=8)
            np.testing.assert_array_equal(bits(got), bits(g["timing_gemv_2880"]))
            checks += columns
            continue
        act = oracle.quantize_q8_0(floats.reshape(8, n)).reshape(-1).copy()
        act[2] = 0x80  # activations[0].qs[0] = -128
        got = oracle.gemv(QUANT_MXFP4, n, w, act[:blocks * 34])
        np.testing.assert_array_equal(bits(got), bits(g[f"gemv_{n}_{columns}"]))
        checks += columns
        act = oracle.quantize_q8_0(floats.reshape(8, n))
        for rows in (4, 8):
            stride = columns + 3
            exp = g[f"gemm_{n}_{columns}_{rows}"].reshape(rows, stride)
            for r in range(rows):
                got = oracle.gemv(QUANT_MXFP4, n, w, act[r])
                np.testing.assert_array_equal(bits(got), bits(exp[r, :columns]))
            assert np.all(exp[:, columns:] == np.float32(-123.25)), "stride canary overwritten"
            checks += rows * columns
    assert h.digest() == bytes(g["inputs_sha256"]), "replayed mt19937 inputs drifted"
    assert checks == 2880 + 3 * (8 + 16 + 64) * 13


def test_compatible_down_golden(oracle, golden_dir):
    """hybrid_layer.cpp:964-979 adversarial bank x sine / zero / q8-ties (bitwise, test_compatible_down.py)."""
    g = np.load(os.path.join(golden_dir, "compatible_down.npz"))
    w = compatible_weights()
    np.testing.assert_array_equal(w, g["weights"])
    for pattern in ("sine", "zero", "q8-ties"):
        for sample in range(3):
            act, exp = g[f"{pattern}_{sample}_act"], g[f"{pattern}_{sample}_out"]
            for j in range(act.shape[0]):
                e = j % 4
                got = oracle.gemv(QUANT_MXFP4, 128, w[e * 64 * 4:(e + 1) * 64 * 4], act[j])
                np.testing.assert_array_equal(bits(got), bits(exp[j]))


def test_q8_ties_quantizer(oracle):
    """The q8-ties activations (hybrid_layer.cpp:598-601) hit exact half-way codes: rn-even."""
    v = activation_input(128 * 4, 1, "q8-ties")
    q = oracle.quantize_q8_0(v.reshape(-1, 128)).reshape(-1, 34)
    for b in range(q.shape[0]):
        blk = v[b * 32:(b + 1) * 32]
        amax = np.max(np.abs(blk))
        assert amax == 127.0
        codes = q[b, 2:].view(np.int8).astype(np.int64)
        np.testing.assert_array_equal(codes, np.rint(blk).astype(np.int64))  # numpy rint is half-even
        d = q[b, :2].view(np.float16)[0]
        assert d == np.float16(np.float32(127.0) / np.float32(127.0))


def test_quantized_down_golden(oracle, golden_dir):
    """tests/test_quantized_cuda.cpp:31-41 samples incl. zero input and 0x80 in every block."""
    g = np.load(os.path.join(golden_dir, "quantized_down.npz"))
    w, jobs = g["weights"], g["jobs"]
    regen = oracle.gen_mxfp4(4170, 1, 0, w.shape[0]).reshape(w.shape)
    np.testing.assert_array_equal(regen, w)
    for s in range(12):
        act, exp = g[f"s{s}_act"], g[f"s{s}_out"]
        if s == 11:
            assert np.all(act.reshape(-1)[2::34] == 0x80)
        if s == 0:
            assert np.all(exp == 0)
        for j, (_, _, e) in enumerate(jobs):
            got = oracle.gemv(QUANT_MXFP4, 128, w[e * 64 * 4:(e + 1) * 64 * 4], act[j])
            np.testing.assert_array_equal(bits(got), bits(exp[j]))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_dequant_matches_gguf(oracle, seed):
    """MXFP4 and Q8_0 dequantisation equal gguf-py's (bit-exact dequant gate)."""
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as QT
    from gguf.quants import dequantize
    mx = oracle.gen_mxfp4(seed, 7, 0, 256, e_lo=0, e_span=256)
    got = oracle.dequant(QUANT_MXFP4, mx, 256 * 32)
    ref = dequantize(mx.reshape(1, -1), QT.MXFP4).reshape(-1).astype(np.float32)
    np.testing.assert_array_equal(bits(got), bits(ref))
    q8 = oracle.gen_q8_0(seed, 8, 0, 256)
    got = oracle.dequant(8, q8, 256 * 32)
    ref = dequantize(q8.reshape(1, -1), QT.Q8_0).reshape(-1).astype(np.float32)
    np.testing.assert_array_equal(bits(got), bits(ref))


def test_oracle_nan_logits_pick_lowest_experts(oracle):
    """NaN logits rank lowest: a token whose logits are all NaN goes to experts 0..k-1."""
    from tests.helpers import host_weights, oracle_desc, small_config
    cfg = small_config()
    w = host_weights(oracle, cfg)
    x = np.ones((2, cfg.hidden), np.float32)
    x[0, 5] = np.nan
    ids, _, _ = oracle.route(oracle_desc(cfg), w, x)
    np.testing.assert_array_equal(ids[0], np.arange(cfg.top_k))
    assert ((ids[1] >= 0) & (ids[1] < cfg.experts)).all()
