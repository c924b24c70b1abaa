"""GPU parity of the kernels behind the C ABI against the CPU oracle:
block dequant bit-exact for every format, the quantised matvec within the
GEMV tolerance on every format and on the microbenchmark shapes."""
import numpy as np
import pytest
from conftest import bits_equal

from distcomp_b200 import gguf as G

pytestmark = pytest.mark.gpu

ALL_TYPES = [G.F32, G.F16, G.Q4_0, G.Q4_1, G.Q5_0, G.Q5_1, G.Q8_0, G.Q2_K, G.Q3_K, G.Q4_K, G.Q5_K,
             G.Q6_K, G.Q8_K]


def test_dequant_fixture_blocks_bit_exact(eng, golden):
    """The reference decoder's output on random blocks (fp16 NaN/inf/subnormal
    scales included) is reproduced bit for bit on the device."""
    d = golden("dequant_blocks.npz")
    for t in sorted({int(k.split("_")[1]) for k in d if k.startswith("raw_")}):
        total, n = (int(v) for v in d[f"n_{t}"])
        rc, got = eng.dequant(t, d[f"raw_{t}"], total, 0, n)
        assert rc == 0, t
        assert bits_equal(got, d[f"out_{t}"]), f"type {t}"


@pytest.mark.parametrize("t", ALL_TYPES)
def test_dequant_ranges_bit_exact(eng, oracle_port, t):
    rng = np.random.default_rng(t + 11)
    be, bb = (1, 4) if t == G.F32 else (1, 2) if t == G.F16 else G.BLOCK[t]
    nblk = 300
    total = nblk * be if be > 1 else 4096
    raw = rng.integers(0, 256, size=total * bb // be + 64, dtype=np.uint8)
    if t == G.F32:   # keep F32 payloads finite-ish (NaN bit patterns compare by bits anyway)
        pass
    cases = [(0, total - (be if t == G.Q8_K else 0))]
    step = be if be > 1 else 1
    cases += [(step * 5, step * 17 + (3 if be > 1 else 0)), (step * 40, step)]
    for off, n in cases:
        r1, a = eng.dequant(t, raw, total, off, n)
        r2, b = oracle_port.dequant(t, raw, total, off, n)
        assert r1 == r2 == 0
        assert bits_equal(a, b), (t, off, n)


def test_dequant_rejects_like_reference(eng):
    raw = np.zeros(34 * 8, dtype=np.uint8)
    assert eng.dequant(G.Q8_0, raw, 256, 16, 32)[0] == -1
    assert eng.dequant(G.Q8_0, raw, 256, 240, 32)[0] == -1
    assert eng.dequant(G.Q8_1, raw, 256, 0, 32)[0] == -1
    assert eng.dequant(G.Q8_0, raw, 256, 0, 0)[0] == 0


def gemv_tol_ok(y, ref64, w_norms, x):
    """|y - ref| <= 1e-4 * |ref| + 1e-6 * ||w_o|| * ||x||, ref in double.

    Relative 1e-4 where the row sum is large; where it cancels, an absolute
    floor on the scale of the row (Cauchy-Schwarz bound).  The reference's
    own sequential fp32 matvec is off by up to ~1.6e-7 * ||w_o|| * ||x||
    (16% relative on cancelling rows) on these shapes, so the floor is set a
    few times above that, and every test checks the reference's fp32 result
    against the same bound."""
    bound = 1e-4 * np.abs(ref64) + 1e-6 * w_norms * np.linalg.norm(x.astype(np.float64))
    err = np.abs(y.astype(np.float64) - ref64)
    return bool(np.all(err <= bound)), float(np.max(err / (np.abs(ref64) + 1e-30)))


def row_norms(oracle_port, t, raw, n_in, n_out):
    total = n_in * n_out
    rc, w = oracle_port.dequant(t, raw, total, 0, total)
    assert rc == 0
    return np.linalg.norm(w.reshape(n_out, n_in).astype(np.float64), axis=1)


def random_weights(rng, t, n_in, n_out):
    if t == G.F32:
        return (rng.standard_normal(n_in * n_out).astype(np.float32) * 0.02).view(np.uint8)
    if t == G.F16:
        return (rng.standard_normal(n_in * n_out).astype(np.float16) * np.float16(0.02)).view(np.uint8)
    from distcomp_b200 import synth
    if t in (G.Q4_0, G.Q4_1, G.Q5_0, G.Q5_1, G.Q8_0):
        w = rng.standard_normal((n_out, n_in)).astype(np.float32) * np.float32(0.02)
        return synth.quantize_numpy(w, t)
    be = G.BLOCK[t][0]
    return synth.random_kquant_blocks(rng, t, n_in * n_out // be)


@pytest.mark.parametrize("t", [G.F32, G.F16, G.Q4_0, G.Q4_1, G.Q5_0, G.Q5_1, G.Q8_0, G.Q2_K, G.Q3_K,
                               G.Q4_K, G.Q5_K, G.Q6_K])
@pytest.mark.parametrize("n_in,n_out", [(256, 96), (1024, 200), (2048, 333)])
def test_matvec_formats(eng, oracle_port, t, n_in, n_out):
    rng = np.random.default_rng(n_in * 7 + t)
    raw = random_weights(rng, t, n_in, n_out)
    x = rng.standard_normal(n_in).astype(np.float32)
    y = eng.matvec(t, raw, n_in, n_out, x)
    ref = oracle_port.matvec_f64(t, raw, n_in, n_out, x)
    ok, worst = gemv_tol_ok(y, ref, row_norms(oracle_port, t, raw, n_in, n_out), x)
    assert ok, f"type {t} {n_out}x{n_in}: worst rel {worst:.3e}"
    # the reference's own fp32 result is within the same band
    y32 = oracle_port.matvec(t, raw, n_in, n_out, x)
    assert gemv_tol_ok(y32, ref, row_norms(oracle_port, t, raw, n_in, n_out), x)[0]


def test_matvec_zero_rule(eng, oracle_port):
    """A quantised tensor whose n_in is not a whole number of blocks gives
    zeros, as the reference's matvec does (src/engine.c:317-320)."""
    rng = np.random.default_rng(3)
    n_in, n_out = 48, 20
    raw = rng.integers(0, 256, size=34 * 2 * n_out, dtype=np.uint8)
    x = rng.standard_normal(n_in).astype(np.float32)
    assert np.all(eng.matvec(G.Q8_0, raw, n_in, n_out, x) == 0)
    assert np.all(oracle_port.matvec(G.Q8_0, raw, n_in, n_out, x) == 0)


def microbench_weights(rng, t, n_in, n_out):
    """Codes uniform over the format's range, fp16 scales |N(0,0.02)|/max_code."""
    from distcomp_b200 import synth
    return synth.microbench_blocks(rng, t, n_in, n_out)


@pytest.mark.parametrize("t", [G.Q4_0, G.Q8_0])
@pytest.mark.parametrize("n_out,n_in", [(4096, 4096), (14336, 4096), (4096, 14336)])
def test_matvec_microbench_shapes(eng, oracle_port, t, n_out, n_in):
    """The GEMV microbenchmark shapes through the fast path, against the
    double-precision oracle with the microbenchmark's tolerance."""
    rng = np.random.default_rng(n_out + n_in + t)
    raw = microbench_weights(rng, t, n_in, n_out)
    x = rng.standard_normal(n_in).astype(np.float32)
    y = eng.matvec(t, raw, n_in, n_out, x)
    ref = oracle_port.matvec_f64(t, raw, n_in, n_out, x)
    wn = row_norms(oracle_port, t, raw, n_in, n_out)
    ok, worst = gemv_tol_ok(y, ref, wn, x)
    assert ok, f"worst rel {worst:.3e}"
    assert gemv_tol_ok(oracle_port.matvec(t, raw, n_in, n_out, x), ref, wn, x)[0]


@pytest.mark.parametrize("t", [G.Q4_0, G.Q8_0, G.Q4_K])
def test_matvec_streamed_phases(eng, oracle_port, t):
    """The streamed microbenchmark (copies as GEMV phases of one persistent
    launch): the last phase's y against the double-precision oracle, and a
    matrix without a fast layout refused with a message."""
    rng = np.random.default_rng(40 + t)
    n_in, n_out = 4096, 1536
    raw = microbench_weights(rng, t, n_in, n_out) if t != G.Q4_K else random_weights(rng, t, n_in, n_out)
    x = rng.standard_normal(n_in).astype(np.float32)
    ms, y = eng.matvec_stream_bench(t, raw, n_in, n_out, x, copies=3, rounds=2)
    assert ms > 0
    ref = oracle_port.matvec_f64(t, raw, n_in, n_out, x)
    ok, worst = gemv_tol_ok(y, ref, row_norms(oracle_port, t, raw, n_in, n_out), x)
    assert ok, f"worst rel {worst:.3e}"
    raw2 = microbench_weights(rng, G.Q4_0, 512, 64)
    with pytest.raises(eng.EngineError, match="fast layout"):
        eng.matvec_stream_bench(G.Q4_0, raw2, 512, 64, x[:512], copies=2, rounds=1)


def test_matvec_extreme_inputs(eng, oracle_port):
    """Large/small dynamic range in x (digit decomposition edge cases) and
    all-zero blocks."""
    rng = np.random.default_rng(5)
    n_in, n_out = 2048, 64
    raw = microbench_weights(rng, G.Q4_0, n_in, n_out)
    for x in (rng.standard_normal(n_in).astype(np.float32) * 1e4,
              rng.standard_normal(n_in).astype(np.float32) * 1e-6,
              np.where(rng.random(n_in) < 0.5, 0, rng.standard_normal(n_in)).astype(np.float32),
              np.concatenate([np.zeros(1024), rng.standard_normal(1024) * 300]).astype(np.float32),
              np.full(n_in, 127.5, dtype=np.float32)):
        y = eng.matvec(G.Q4_0, raw, n_in, n_out, x)
        ref = oracle_port.matvec_f64(G.Q4_0, raw, n_in, n_out, x)
        ok, worst = gemv_tol_ok(y, ref, row_norms(oracle_port, G.Q4_0, raw, n_in, n_out), x)
        assert ok, worst


@pytest.mark.parametrize("t", [G.Q4_0, G.Q8_0, G.Q4_K])
@pytest.mark.parametrize("n_out,n_in", [(1024, 8192), (512, 28672)])
def test_matvec_fast_widths(eng, oracle_port, t, n_out, n_in):
    """Q4_K rows through the SPLITK4 fast GEMV; 28672 inputs (the 70B-shape
    ffn_down width, above one 16384-input column segment) stored as two
    segments whose GEMVs store and then add."""
    rng = np.random.default_rng(n_out + n_in + 3 * t)
    raw = random_weights(rng, t, n_in, n_out)
    x = rng.standard_normal(n_in).astype(np.float32)
    y = eng.matvec(t, raw, n_in, n_out, x)
    ref = oracle_port.matvec_f64(t, raw, n_in, n_out, x)
    ok, worst = gemv_tol_ok(y, ref, row_norms(oracle_port, t, raw, n_in, n_out), x)
    assert ok, f"type {t} {n_out}x{n_in}: worst rel {worst:.3e}"
