// Exchanges of the tensor-parallel batched prefill (tp_prefill.cu).
#pragma once

#include "gemv.cuh"

namespace tvb {

// Floats of one prefill region (a multiple of 64): `rows` partial rows of H,
// then `rows` per-row partial sums of squares.  Each rank has two.
size_t tp_prefill_region_floats(int rows, int H);

// Flag sync of all ranks (one more exchange number in st->tp_epoch).
tvb_status tp_sync(const TpArgs& t, StepState* st, cudaStream_t stream, bool pdl = false);
// x [S][H] += inv_rms * sum of every rank's partial rows in the region at
// float offset `off` (rows [S][H], then the S sums of squares of a sub-norm of
// full length norm_n; norm_n == 0: no sub-norm).
tvb_status tp_reduce_rows(const TpArgs& t, size_t off, int S, int H, int norm_n, float eps, float* x,
                          cudaStream_t stream, bool pdl = false);

}  // namespace tvb
