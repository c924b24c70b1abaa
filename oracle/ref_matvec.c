/*
 * ref_matvec.c -- the REFERENCE's quantised matvec alone, for timing.
 *
 * TEST INFRASTRUCTURE ONLY.  The reference keeps matvec() file-static in
 * src/engine.c:348-357 (rows split over its thread pool, src/thread.c:204-237;
 * each row decoded and accumulated by matvec_range, src/engine.c:287-343), so
 * this translation unit includes that file where it lies (never a copy) and
 * exports one wrapper.  oracle/Makefile links it with src/gguf.c, thread.c
 * and util.c into oracle/_ref/libdcref_mv.so; bench.py's GEMV microbenchmark
 * times it on the host cores as the CPU baseline.
 */
#include "engine.c"

void refmv_set_threads(int n) { tp_set(n); }

/* y = W x for `n_out` rows of `n_in` inputs of raw GGUF blocks of type t. */
int refmv_matvec(unsigned t, const void *raw, size_t nbytes, int n_in, int n_out, const float *x, float *y)
{
    gguf_tensor w;
    memset(&w, 0, sizeof w);
    w.type = t;
    w.n_dims = 2;
    w.dims[0] = (unsigned long)n_in;
    w.dims[1] = (unsigned long)n_out;
    w.data = (const unsigned char *)raw;
    w.nbytes = nbytes;
    matvec(y, &w, x, n_in, n_out);
    return 0;
}
