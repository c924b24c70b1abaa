"""The synthetic-model generators: the torch quantisers against gguf-py's
numpy rule (bit-identical bytes) and the Q4_K quantiser's blocks decoded by
the oracle and by the reference's own decoder (oracle/_ref, when built)."""
import numpy as np
import pytest
import torch

from distcomp_b200 import gguf as G
from distcomp_b200 import synth


@pytest.mark.parametrize("t", [G.Q4_0, G.Q8_0])
def test_quantize_torch_matches_numpy_rule(t):
    rng = np.random.default_rng(7 + t)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0                       # an all-zero block
    w[5, 40] = 0.5                        # a block with one large element
    w[7, 35], w[7, 50] = -0.25, 0.25      # the block maximum twice, opposite signs: the first decides
    w[9, 70], w[9, 66] = 0.25, -0.25
    a = synth.quantize_numpy(w, t)
    b = synth.quantize_torch(torch.from_numpy(w.reshape(-1)), t).numpy()
    assert np.array_equal(a, b)


def q4k_case():
    rng = np.random.default_rng(11)
    w = (rng.standard_normal(256 * 96) * 0.02).astype(np.float32)
    w[:256] = 0.0                         # all-zero super-block: d = dmin = 0
    w[256:288] = -0.03                    # a negative-only sub-block
    return w, synth.quantize_q4_k_torch(torch.from_numpy(w)).numpy()


def test_q4_k_quantiser_blocks_decode_to_the_weights(oracle_port):
    w, qb = q4k_case()
    assert qb.size == w.size // 256 * 144
    rc, y = oracle_port.dequant(G.Q4_K, qb, w.size, 0, w.size)
    assert rc == 0
    assert np.all(y[:256] == 0.0)
    # within half a code step of each sub-block (range / 15, a little more
    # for the 6-bit scale's rounding) plus half a step of the 6-bit minimum
    # (dmin = the super-block's largest minimum / 63)
    W = w.reshape(-1, 32)
    lo = np.minimum(W.min(1), 0)
    step = (W.max(1) - lo) / 15
    dmin = np.repeat((-lo).reshape(-1, 8).max(1) / 63, 8)
    err = np.abs(y - w).reshape(-1, 32).max(1)
    assert np.all(err <= 0.51 * step + 0.5 * dmin + 1e-6)
    assert np.corrcoef(y[256:], w[256:])[0, 1] > 0.99


def test_q4_k_quantiser_blocks_reference_decoder(oracle_port, oracle_ref):
    w, qb = q4k_case()
    rc, y = oracle_port.dequant(G.Q4_K, qb, w.size, 0, w.size)
    rc2, y2 = oracle_ref.dequant(G.Q4_K, qb, w.size, 0, w.size)
    assert rc == rc2 == 0 and np.array_equal(y.view(np.uint32), y2.view(np.uint32))


def test_q4k_specs():
    s = synth.spec("wide-q4k")
    assert s.wtype == G.Q4_K and s.n_ff > 16384 and s.n_ff % 2048 == 0
    assert all(gt == G.Q4_K for name, dims, gt in synth.tensor_list(s) if name.startswith("blk.")
               and name.endswith("weight") and "norm" not in name)


@pytest.mark.gpu
@pytest.mark.parametrize("t", [G.Q4_0, G.Q8_0])
def test_quantize_torch_on_gpu_matches_numpy_rule(t):
    """The same bytes on the GPU, with many blocks whose maximum magnitude
    occurs twice with opposite signs (the first one decides a Q4_0 block)."""
    rng = np.random.default_rng(17 + t)
    w = (rng.standard_normal((4096, 256)) * 0.02).astype(np.float32)
    blk = w.reshape(-1, 32)
    for i in range(0, blk.shape[0], 3):
        j = int(np.argmax(np.abs(blk[i])))
        blk[i, (j + 1 + i % 31) % 32] = -blk[i, j]
    a = synth.quantize_numpy(w, t)
    b = synth.quantize_torch(torch.from_numpy(w.reshape(-1)).cuda(), t).cpu().numpy()
    assert np.array_equal(a, b)
