"""The no-allocation logits+argmax entry point against the allocating one.

ecu_matvec_argmax_noalloc exists for callers that cannot allocate device
memory (a node held to a fixed memory budget, a host with its own device
pool, a loop that cannot take cudaMalloc's synchronisation): it works on
device buffers the caller owns and keeps its scratch in a fixed array inside
the library.  This file is collected last so that a failure here leaves
every other test already run; it passes alone or after them."""
import numpy as np
import pytest

from distcomp_b200 import gguf as G
from distcomp_b200 import synth

pytestmark = pytest.mark.gpu

LIMIT_ROWS = 524288


def first_max(y: np.ndarray) -> int:
    """llm_pick's rule (src/engine.c:517-526): first maximum, strict >."""
    best, bv = 0, y[0]
    for i in range(1, len(y)):
        if y[i] > bv:
            best, bv = i, y[i]
    return best


def weights(rng, t, n_in, n_out):
    w = (rng.standard_normal((n_out, n_in)) * 0.02).astype(np.float32)
    return synth.quantize_numpy(w, t)


@pytest.mark.parametrize("t,n_in,n_out", [(G.Q8_0, 4096, 5000), (G.Q4_0, 4096, 1024 + 77), (G.F32, 688, 300)])
def test_noalloc_matches_matvec_twice(eng, oracle_port, t, n_in, n_out):
    import torch
    L = eng.lib()
    rng = np.random.default_rng(n_out)
    raw = weights(rng, t, n_in, n_out)
    x = rng.standard_normal(n_in).astype(np.float32)
    y_alloc = eng.matvec(t, raw, n_in, n_out, x).astype(np.float64)   # the allocating entry point
    y_ref = oracle_port.matvec_f64(t, raw, n_in, n_out, x).astype(np.float64)   # the oracle, in double
    rc, w = oracle_port.dequant(t, raw, n_in * n_out, 0, n_in * n_out)
    assert rc == 0
    wn = np.linalg.norm(w.reshape(n_out, n_in).astype(np.float64), axis=1)
    bound = 1e-4 * np.abs(y_ref) + 2e-6 * wn * np.linalg.norm(x.astype(np.float64))
    assert np.all(np.abs(y_alloc - y_ref) <= bound)
    tok_ref = first_max(y_ref)
    dev = torch.device("cuda:0")
    d_w = torch.from_numpy(raw).to(dev)
    d_x = torch.from_numpy(x).to(dev)
    d_y = torch.empty(n_out, dtype=torch.float32, device=dev)
    d_tok = torch.empty(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):                     # the second call reuses the scratch
        d_y.fill_(float("nan"))
        d_tok.fill_(-7)
        rc = L.ecu_matvec_argmax_noalloc(t, d_w.data_ptr(), n_in, n_out, d_x.data_ptr(), d_y.data_ptr(),
                                         d_tok.data_ptr(), stream)
        assert rc == 0, eng.last_error()
        torch.cuda.synchronize(dev)
        y = d_y.cpu().numpy().astype(np.float64)
        tok = int(d_tok.cpu()[0])
        for ref, what in ((y_ref, "oracle"), (y_alloc, "ecu_matvec")):
            err = np.abs(y - ref)
            assert np.all(err <= bound), f"call {call} vs {what}: worst {np.max(err / bound):.2f} of the bound"
        assert tok == first_max(d_y.cpu().numpy()), f"call {call}"
        # the oracle's token, unless its two best logits are closer than the
        # tolerance (then either is a correct first maximum)
        srt = np.sort(y_ref)
        if srt[-1] - srt[-2] > 2 * bound[tok_ref]:
            assert tok == tok_ref, f"call {call}: token {tok} != oracle {tok_ref}"


def test_noalloc_rejects_oversize(eng):
    import torch
    L = eng.lib()
    dev = torch.device("cuda:0")
    d = torch.zeros(64, dtype=torch.float32, device=dev)
    tok = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = L.ecu_matvec_argmax_noalloc(G.Q8_0, d.data_ptr(), 32, LIMIT_ROWS + 1, d.data_ptr(), d.data_ptr(),
                                     tok.data_ptr(), None)
    assert rc == -1
    assert "exceeds the no-allocation limit" in eng.last_error()
