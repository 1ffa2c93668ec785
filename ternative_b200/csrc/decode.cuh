// The whole decode step (Model::forward_gpu, src/model.cpp:1354-1582) as one
// persistent kernel: one CTA of 16 warps per SM, launched cooperatively so all
// CTAs are resident, walking a table of phases
//
//   per layer: QKV+RoPE+KV append | attention | sub-norm+o_proj+residual |
//              ffn_norm+gate/up+relu^2*up | sub-norm+down+residual
//   then:      output_norm + lm_head + argmax
//
// separated by grid-wide barriers.  Before a CTA enters a barrier its warps
// have already requested their first weight chunks of the next phase (weights
// do not depend on the barrier), so HBM keeps streaming while the grid
// synchronises and the next phase's activations are being read.
//
// Every spin is bounded: a barrier that waits about a second sets the abort
// flag and the timeout status, and every CTA then leaves at its next barrier.
#pragma once

#include "attention.cuh"
#include "attn_split.cuh"

namespace tvb {

enum PhaseKind { PK_GEMV = 0, PK_ATTN = 1 };

struct alignas(16) Phase {
    int kind;   // PhaseKind
    int mode;   // GemvMode (PK_GEMV)
    int wt;     // WType (PK_GEMV)
    GemvArgs g;
    AttnArgs at;
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier, split so a CTA can do input-independent work between its
// arrival and its wait.  Arrival: release-add on the counter (no round trip).
__device__ __forceinline__ void grid_arrive(StepState* st) {
    __syncthreads();
    if (threadIdx.x == 0)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&st->bar_ctr) : "memory");
}

// Wait until `target` arrivals (barrier n of this launch: n * gridDim.x).
// Returns false on abort or after ~1 s (then sets abort and the timeout bit).
// The poll is a single acquire load per round (the abort latch and the clock
// are looked at every 32 rounds): a second dependent load per round doubled
// the time to notice the last arrival (measured: 51 us per 2B step).  The
// acquire orders this thread after every arriver's release; the
// __syncthreads passes that on to the CTA.
__device__ __forceinline__ bool grid_wait(StepState* st, unsigned target) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        int ok = 1;
        const long long t0 = clock64();
        unsigned it = 0;
        while (ld_acquire_gpu(&st->bar_ctr) < target) {
            if ((++it & 31u) != 0) continue;
            if (ld_acquire_gpu(&st->abort)) {
                ok = 0;
                break;
            }
            if (clock64() - t0 > kSpinLimitCycles) {
                atomicOr(&st->abort, 1u);
                atomicOr(&st->status, kStatusTimeout);
                ok = 0;
                break;
            }
        }
        s_ok = ok;
    }
    trace_stamp(7);   // (thread 0: its poll saw the last arrival)
    __syncthreads();
    return s_ok != 0;
}

// End of a row-parallel phase under tensor parallelism (exchange n): every CTA
// of every rank has set its flag slot on this rank (warp 0 watches them).
__device__ __forceinline__ bool tp_exchange_wait(StepState* st, const TpArgs& t, unsigned n, int G) {
    __shared__ int s_tp_ok;
    if (threadIdx.x < 32) {
        const bool ok = tp_flag_wait(t, n, G, &st->abort, &st->status);
        if (threadIdx.x == 0) s_tp_ok = ok ? 1 : 0;
    }
    __syncthreads();
    return s_tp_ok != 0;
}

#define TVB_GEMV_CASES(X)                                                     \
    X(GM_QKV, WT_F16, 2) X(GM_QKV, WT_I8, 2) X(GM_RESID, WT_F16, 1)           \
    X(GM_RESID, WT_I8, 1) X(GM_GATEUP, WT_F16, 2) X(GM_GATEUP, WT_I8, 2)      \
    X(GM_LMHEAD, WT_F16, 1)

// Input-independent work for a phase: stage its constants (norm weight, row
// scales, RoPE row) in shared memory, then request its first weight chunks.
// In this order the staging loads return before the chunk requests fill the
// SM's load path (the reverse measured 54 us per 2B step slower together with
// the poller's own staging).
__device__ __forceinline__ void phase_prepare(const Phase& ph, unsigned char* smem, int G, int b, int warp,
                                             int pos, ChunkBuf& buf) {
    if (ph.kind != PK_GEMV) return;
#define X(M, W, R)                                          \
    if (ph.mode == M && ph.wt == W) {                       \
        gemv_stage<M, W, R>(ph.g, smem, G, pos);            \
        gemv_prefetch<M, W, R>(ph.g, G, b, warp, buf);      \
        return;                                             \
    }
    TVB_GEMV_CASES(X)
#undef X
}

template <bool TP>
__device__ __forceinline__ void phase_gemv(const Phase& ph, unsigned char* smem, int G, int pos, int token,
                                           ChunkBuf& buf, GemvArgmax& best, unsigned push0) {
#define X(M, W, R)                                                                \
    if (ph.mode == M && ph.wt == W) {                                             \
        gemv_run<M, W, R, TP>(ph.g, smem, G, pos, token, buf, best, push0);       \
        return;                                                                   \
    }
    TVB_GEMV_CASES(X)
#undef X
}

// Copy a phase descriptor into shared memory (all threads, 16-byte words).
__device__ __forceinline__ void load_phase(Phase* dst, const Phase* src) {
    const int4* s4 = reinterpret_cast<const int4*>(src);
    int4* d4 = reinterpret_cast<int4*>(dst);
    for (int i = threadIdx.x; i < (int)(sizeof(Phase) / 16); i += blockDim.x) d4[i] = __ldg(s4 + i);
}

// Shared memory of the step kernel: [0, 1024) two phase descriptors (double
// buffered), then the per-phase layouts (gemv_smem_layout / attention scratch).
static_assert(2 * sizeof(Phase) <= 1024, "phase descriptors must fit the reserved area");

// Tensor parallelism (TP instantiation): n_push row-parallel exchanges and
// n_argmax (0 or 1) argmax exchanges in the phase table.
template <bool TP>
__global__ void __launch_bounds__(kGemvThreads, 1)
decode_step_kernel(const Phase* __restrict__ phases, int n_phases, StepState* st, int n_push, int n_argmax) {
    extern __shared__ __align__(128) unsigned char smem[];
    Phase* desc = reinterpret_cast<Phase*>(smem);   // desc[p & 1]
    const int warp = threadIdx.x >> 5;
    const int G = gridDim.x, b = blockIdx.x;
    // the step's position and token are fixed until the lm_head's last CTA
    // advances them at the very end
    const int pos = __ldcg(&st->pos);
    const int token = __ldcg(&st->token);
    const unsigned epoch0 = __ldcg(&st->tp_epoch);
    const unsigned push0 = __ldcg(&st->tp_pushes);

    ChunkBuf buf;
    load_phase(&desc[0], &phases[0]);
    __syncthreads();
    phase_prepare(desc[0], smem, G, b, warp, pos, buf);
    __syncthreads();
    bool ok = true;
    for (int p = 0; p < n_phases && ok; ++p) {
#ifdef TVB_PHASE_TRACE
        if (threadIdx.x == 0)
            s_trace_row = (g_trace_buf && p < g_trace_phases) ? g_trace_buf + ((size_t)p * G + b) * kTraceEvents
                                                              : nullptr;
#endif
        trace_stamp(0);
        const Phase& ph = desc[p & 1];
        // The next phase's descriptor.  Its buffer held phase p - 1, which
        // nothing reads any more; the GEMV prologue's __syncthreads (or the
        // one below) publishes it.
        const Phase& next = desc[(p + 1) & 1];
        if (p + 1 < n_phases) load_phase(&desc[(p + 1) & 1], &phases[p + 1]);
        const bool exchange =
            TP && ph.kind == PK_GEMV && ph.mode == GM_RESID && ph.g.tp.world > 1 && ph.g.tp.index >= 0;
        const TpArgs& tp = ph.g.tp;
        if (ph.kind == PK_GEMV) {
            GemvArgmax best{-INFINITY, 0};
            phase_gemv<TP>(ph, smem, G, pos, token, buf, best, push0);
            if (ph.mode == GM_LMHEAD) lmhead_finish<TP>(ph.g, best, epoch0);
        } else {
            // No weight chunks are in flight across an attention phase (it has
            // none to prefetch); saying so frees the chunk registers for it.
            buf = ChunkBuf{};
            __syncthreads();
            if (b < ph.at.nkv * ph.at.nsplit) attn_item(ph.at, b, smem + 1024, pos);
            trace_stamp(1);
        }
        // A row-parallel exchange is waited for even after the last phase: the
        // next launch's first exchange reuses this one's slot parity.
        if (p + 1 < n_phases || exchange) {
            grid_arrive(st);   // this phase's outputs are written (includes __syncthreads)
            if (exchange && threadIdx.x == 0) tp_flag_arrive(tp, push0 + (unsigned)tp.index + 1u);
            trace_stamp(6);
            // input-independent work for the next phase overlaps the barrier
            if (p + 1 < n_phases) phase_prepare(next, smem, G, b, warp, pos, buf);
            trace_stamp(4);
            ok = exchange ? tp_exchange_wait(st, tp, push0 + (unsigned)tp.index + 1u, G)
                          : grid_wait(st, (unsigned)(p + 1) * (unsigned)G);
            trace_stamp(5);
        }
    }
    // last CTA out resets the barrier for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&st->exit_ctr, 1u) == (unsigned)G - 1u) {
            st->bar_ctr = 0u;
            st->exit_ctr = 0u;
            st->tp_epoch = epoch0 + (unsigned)n_argmax;
            st->tp_pushes = push0 + (unsigned)n_push;
            __threadfence();
        }
    }
}

}  // namespace tvb
