"""The oracle pinned against the reference's own outputs (CPU only).

Fixtures in tests/golden/ were produced by importing the reference's golden.py
and rounding.py unmodified (tests/golden/make_fixtures.py). Every comparison
against them here is bit-exact, except where scipy's erf stands in for libm's.
"""

import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import golden as O
from tfb200 import workloads as W

GOLDEN = Path(__file__).resolve().parent / "golden"


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


# ------------------------------------------------------------------ rounding pins


def test_to_bf16_matches_reference_on_consistency_vector():
    r = np.load(GOLDEN / "rounding_vectors.npz")
    cons = O.lcg_u32(1000, 0x5EED2026)
    assert np.array_equal(cons, r["consistency_in"])  # the LCG itself (rounding.py:125-137)
    got = bits(O.to_bf16(cons.view(np.float32)))
    assert np.array_equal(got, r["consistency_out"])


def test_to_bf16_matches_reference_on_special_values():
    r = np.load(GOLDEN / "rounding_vectors.npz")
    got = bits(O.to_bf16(r["specials_in"].view(np.float32)))
    assert np.array_equal(got, r["specials_out"])


@pytest.mark.parametrize("inp,want", [
    (0x3F808000, 0x3F800000),   # tie -> even, rounds down (test_rounding.py:62-66)
    (0x3F818000, 0x3F820000),   # tie -> even, rounds up   (test_rounding.py:69-73)
    (0x7F800000, 0x7F800000),   # +inf
    (0xFF800000, 0xFF800000),   # -inf
    (0x80000000, 0x80000000),   # -0
    (0x7FC00123, 0x7FC00000),   # NaN -> canonical quiet NaN
    (0xFFC00001, 0xFFC00000),   # negative NaN keeps its sign
])
def test_to_bf16_known_answers(inp, want):
    x = np.array([inp], dtype=np.uint32).view(np.float32)
    assert int(bits(O.to_bf16(x))[0]) == want


def test_workload_rounding_agrees_with_oracle():
    cons = O.lcg_u32(1000, 0x5EED2026).view(np.float32)
    assert np.array_equal(W.bf16_bits(cons), O.to_bf16_bits(cons))
    assert np.array_equal(bits(W.bf16_to_f32(W.bf16_bits(cons))), bits(O.to_bf16(cons)))


# ---------------------------------------------------------- hand-computed KATs


def test_reference_hand_computed_kats():
    k = np.load(GOLDEN / "kat_vectors.npz")
    # test_golden.py:34-42: rmsnorm [[1,1],[2,2]], gamma [3,1], eps 0 -> [[3,1],[3,1]]
    assert np.array_equal(O.rmsnorm(k["rmsnorm_x"], k["rmsnorm_gamma"], eps=0.0), k["rmsnorm_out"])
    assert np.allclose(k["rmsnorm_out"], [[3, 1], [3, 1]])
    # test_golden.py:45-51: [[19,22],[43,50]]
    assert np.array_equal(O.matmul(k["matmul_a"], k["matmul_b"]), k["matmul_out"])
    assert np.array_equal(k["matmul_out"], np.array([[19, 22], [43, 50]], np.float32))
    # test_golden.py:54-65: gelu(0,1,-1,2) (bit-exact vs the reference's libm loop)
    assert np.array_equal(bits(O.gelu(k["gelu_x"])), bits(k["gelu_out"]))
    assert np.allclose(k["gelu_out"][:4], [0.0, 0.8413447460685429, -0.15865525393145707, 1.9544997361036416],
                       rtol=1e-5, atol=1e-6)


def test_fused_ops_bit_exact_vs_reference_small():
    k = np.load(GOLDEN / "kat_vectors.npz")
    got = O.fused_mlp(k["mlp_x"], k["mlp_gamma"], k["mlp_w1"], k["mlp_b1"], k["mlp_w2"], k["mlp_res"], 1e-6)
    assert np.array_equal(bits(got), bits(k["mlp_out"]))
    got = O.fused_rmsnorm_matmul(k["mlp_x"], k["mlp_gamma"], k["mlp_w1"], 1e-6)
    assert np.array_equal(bits(got), bits(k["frm_out"]))


def test_fused_equals_composed():
    # test_golden.py:97-123: fused == composed bit for bit
    rng = np.random.default_rng(7)
    x = rng.standard_normal((3, 4)).astype(np.float32)
    g = rng.standard_normal(4).astype(np.float32)
    w = rng.standard_normal((4, 5)).astype(np.float32)
    assert np.array_equal(O.fused_rmsnorm_matmul(x, g, w, 1e-6), O.matmul(O.rmsnorm(x, g, 1e-6), w))


def test_golden_holds_fp32_intermediate():
    # test_golden.py:129-154: the normalised row is not bf16-representable
    x = np.array([[1.0, 2.0]], np.float32)
    n = O.rmsnorm(x, np.ones(2, np.float32), 1e-6)
    assert not np.array_equal(O.to_bf16(n), n)


def test_eps_sensitivity():
    x = np.array([[1.0, 2.0]], np.float32)
    g = np.ones(2, np.float32)
    assert not np.array_equal(O.rmsnorm(x, g, 1e-6), O.rmsnorm(x, g, 1e-2))


# ---------------------------------------------------------- workload pins


@pytest.mark.parametrize("name", ["rmsnorm_matmul_small", "matmul_256x512x1024", "matmul_padded", "mlp_block_small"])
def test_generator_and_oracle_bit_exact_small(name, golden_vectors):
    t = W.generate(name)
    for key, v in t.items():
        want = golden_vectors[f"{name}/sha/{key}"].tobytes().hex()
        assert hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest() == want, key
    wl = W.WORKLOADS[name]
    f = W.bf16_to_f32
    rows = golden_vectors[f"{name}/rows"]
    if wl.kind == "matmul":
        a = f(t["a"])
        if rows.size:
            a = a[rows]
        y = O.matmul(a, f(t["b"]))
    elif wl.kind == "fused_rmsnorm_matmul":
        y = O.fused_rmsnorm_matmul(f(t["x"]), f(t["gamma"]), f(t["w"]), wl.eps)
    else:
        x = f(t["x"])
        y = O.fused_mlp(x, f(t["gamma"]), f(t["w1"]), f(t["b1"]), f(t["w2"]), x, wl.eps, "erf")
    assert np.array_equal(bits(y), bits(golden_vectors[f"{name}/golden"]))


def test_gelu_fast_within_ulps_of_libm():
    x = np.linspace(-8, 8, 20001, dtype=np.float32)
    a = O.gelu(x)
    b = O.gelu_fast(x)
    ulp = np.spacing(np.maximum(np.abs(a), 1e-30).astype(np.float32))
    assert np.all(np.abs(a - b) <= 4 * ulp + 1e-37)


def test_gelu_tanh_close_to_erf():
    x = np.linspace(-6, 6, 4001, dtype=np.float32)
    assert np.max(np.abs(O.gelu_tanh(x) - O.gelu(x))) < 1e-3


def test_device_emulation_within_tolerance_small():
    """The kernel's rounding points keep it within the parity bar (unit-RMS max-abs
    2e-2, PCC 0.9999) of the reference golden on the reference's small shapes."""
    from tfb200.metrics import parity

    t = W.generate("rmsnorm_matmul_small")
    f = W.bf16_to_f32
    g = O.fused_rmsnorm_matmul(f(t["x"]), f(t["gamma"]), f(t["w"]), 1e-5)
    e = O.emulate_device_fused_rmsnorm_matmul(f(t["x"]), f(t["gamma"]), f(t["w"]), 1e-5)
    m = parity(e, g)
    assert m["ok"], m
    assert m["max_abs_unit_rms"] > 0  # non-vacuous: the roundings show
    t = W.generate("mlp_block_small")
    x = f(t["x"])
    g = O.fused_mlp(x, f(t["gamma"]), f(t["w1"]), f(t["b1"]), f(t["w2"]), x, 1e-5, "erf")
    e = O.emulate_device_fused_mlp(x, f(t["gamma"]), f(t["w1"]), f(t["b1"]), f(t["w2"]), x, 1e-5, "erf")
    m = parity(e, g)
    assert m["ok"], m


@pytest.mark.parametrize("name", ["qkv_8192x4096x6144"])
def test_oracle_row_sample_bit_exact_large(name, golden_vectors):
    """The full-size QKV workload: generator hashes and the golden rows."""
    t = W.generate(name)
    for key, v in t.items():
        want = golden_vectors[f"{name}/sha/{key}"].tobytes().hex()
        assert hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest() == want, key
    rows = golden_vectors[f"{name}/rows"]
    f = W.bf16_to_f32
    y = O.fused_rmsnorm_matmul(f(t["x"][rows]), f(t["gamma"]), f(t["w"]), 1e-5)
    assert np.array_equal(bits(y), bits(golden_vectors[f"{name}/golden"]))


# ------------------------------------------------ C restatement (EmitHost golden)


@pytest.fixture(scope="module")
def cg():
    import subprocess

    from oracle import c_golden

    if not c_golden.LIB.exists():
        subprocess.run(["make", "-C", str(c_golden.LIB.parents[1])], check=True, capture_output=True)
    return c_golden


def test_c_rounding_matches_reference_vectors(cg):
    r = np.load(GOLDEN / "rounding_vectors.npz")
    for key in ("consistency", "specials"):
        got = bits(cg.bf16_round(r[f"{key}_in"].view(np.float32)))
        assert np.array_equal(got, r[f"{key}_out"]), key


def test_c_emitted_golden_within_bar_of_reference(cg, golden_vectors):
    """The emitted-host golden rounds its intermediates; it must sit inside the
    parity bar of the fp32 reference golden, and differ from it (non-vacuous)."""
    from tfb200.metrics import parity

    f = W.bf16_to_f32
    t = W.generate("rmsnorm_matmul_small")
    y = cg.fused_rmsnorm_matmul_bf16(f(t["x"]), f(t["gamma"]), f(t["w"]), 1e-5)
    m = parity(y, golden_vectors["rmsnorm_matmul_small/golden"])
    assert m["ok"] and m["max_abs_diff"] > 0, m
    t = W.generate("mlp_block_small")
    x = f(t["x"])
    y = cg.mlp_bf16(x, f(t["gamma"]), f(t["w1"]), f(t["b1"]), f(t["w2"]), x, 1e-5, "erf")
    m = parity(y, golden_vectors["mlp_block_small/golden"])
    assert m["ok"] and m["max_abs_diff"] > 0, m
