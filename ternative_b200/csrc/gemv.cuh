// Batch-1 GEMV for the decode path: y[n] = sum_k W[n][k] * x[k] with F16 or
// INT8 weights and F32 activations/accumulation, fused with the prologue and
// epilogue the reference runs as separate kernels around each GEMV
// (src/model.cpp:1399-1451, cuda/ops_cuda.cu:46-158):
//
//   GM_PLAIN   y = W.x (scaled for INT8)                        gemv_d2d(_int8)
//   GM_QKV     rms_norm(x) -> q,k,v rows -> RoPE -> KV append     :1403-1413
//   GM_RESID   rms_norm_sub(in) -> x += W.in                      :1422-1430, :1442-1450
//   GM_GATEUP  rms_norm(x) -> relu(gate)^2 * up                   :1433-1439
//   GM_LMHEAD  rms_norm(x) -> logits + greedy argmax              :1571-1580
//
// B200 mapping.  A persistent grid (one CTA of 16 warps per SM) gives every CTA
// a balanced, contiguous range of output units (a unit is one row, or the two
// rows an epilogue pairs: RoPE halves, gate/up).  The CTA's rows are cut into
// 2 KB chunks and the (row, chunk) items, in row-major order, are split evenly
// over the 16 warps, so every warp streams the same number of bytes from one
// contiguous span of the weight matrix whatever the row length.  A warp keeps
// kDepth chunks in flight in registers with 128-bit streaming loads (one
// 512-byte coalesced request per warp instruction, L1 bypassed): measured on
// this part, plain streaming loads reach a higher fraction of HBM bandwidth
// than shared-memory staging, whose writes would compete with the reads of the
// activation vector for shared-memory bandwidth.  The first chunks of a phase
// are requested before the wait for the phase's inputs (the grid barrier of the
// decode-step kernel, griddepcontrol.wait in stand-alone launches), so the
// weight stream never drains across a phase boundary.  The normalised
// activation vector lives in shared memory; per-(row, chunk) sums go to shared
// memory and are added in chunk order by the epilogue (deterministic).
#pragma once

#include "stream.cuh"

namespace tvb {

enum GemvMode { GM_PLAIN = 0, GM_QKV = 1, GM_RESID = 2, GM_GATEUP = 3, GM_LMHEAD = 4 };

// Phase trace of the decode step, compiled in only with -DTVB_PHASE_TRACE (the
// libtvb200_trace.so build): thread 0 of every CTA writes %globaltimer (ns) at
// fixed points of each phase into the buffer given to tvb_trace_set, laid out
// [phase][CTA][kTraceEvents].  Events: 0 phase start, 1 inputs staged (GEMV
// prologue done / attention item done), 2 weight stream done, 3 epilogue done,
// 6 barrier arrival made, 4 next phase prepared, 7 thread 0's barrier poll
// succeeded, 5 barrier passed (every warp of the CTA past it).
constexpr int kTraceEvents = 8;
#ifdef TVB_PHASE_TRACE
static __device__ unsigned long long* g_trace_buf;
static __device__ int g_trace_phases;
static __shared__ unsigned long long* s_trace_row;   // this CTA's row of the running phase
__device__ __forceinline__ void trace_stamp(int ev) {
    if (threadIdx.x == 0 && s_trace_row) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        s_trace_row[ev] = t;
    }
}
#else
__device__ __forceinline__ void trace_stamp(int) {}
#endif
enum WType { WT_F16 = 0, WT_I8 = 1 };

constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxKvHeads = 64;
constexpr int kMaxAttnSplits = 8;   // attention splits merged by the o_proj prologue

// Device-resident per-context step state (read/written by the fused kernels).
struct StepState {
    int pos;                        // position of the token being decoded
    int token;                      // token being decoded
    unsigned long long argmax_key;  // packed (ordered logit, ~index) running max
    unsigned lm_done;               // lm_head CTAs finished this step
    unsigned status;                // kStatus* bits, sticky
    int next_token;                 // argmax of this step's logits
    float max_logit;
    unsigned attn_done[kMaxKvHeads];
    unsigned bar_ctr;    // grid-barrier arrivals of the running decode-step launch
    unsigned exit_ctr;   // CTAs that left the running launch
    unsigned abort;      // set when a barrier wait gave up; every CTA then leaves
    unsigned tp_epoch;   // tensor parallelism: argmax exchanges completed so far
    unsigned tp_pushes;  // tensor parallelism: row-parallel exchanges completed so far
};

// Tensor parallelism (one rank per GPU).  Every rank owns an exchange buffer
// that its peers write over NVLink (peer pointers from CUDA IPC):
//   [0, 8)      flags: flags[src] = number of the last argmax exchange rank src
//               signalled
//   [64, 80)    argmax keys of the lm_head slices (64-bit, keys[src])
//   [128, ...)  two slots (exchange number parity) of world x ld floats:
//               slot[src] holds rank src's partial output rows and, at [H],
//               its partial sum of squares of the sub-norm input
//   [xf_off, +world * kTpMaxGrid)  row-exchange flags, one per (rank, CTA):
//               xflags[src][cta] = number of the last row-parallel exchange
//               whose partial rows CTA cta of rank src has written here
constexpr int kMaxTp = 8;
constexpr int kTpFlags = 0, kTpKeys = 64, kTpSlots = 128;
constexpr int kTpMaxGrid = 256;   // flag slots per rank (CTAs of the decode step)

// A zero-initialised TpArgs (world 0) means no tensor parallelism.
struct TpArgs {
    float* peer[kMaxTp];  // every rank's exchange buffer (this rank's at [rank])
    int world, rank;
    int ld;               // floats per rank in a slot (H + 4)
    int index;            // >= 0: row-parallel exchange `index` of the launch (o_proj, down),
                          // or the lm_head's argmax exchange
    int fold;             // >= 0: input = residual + sum of exchange `fold`'s partials
    int norm_n;           // fold: full length of the sub-norm whose partials arrive
    float* x_out;         // fold: where the folded residual is stored (CTA-partitioned)
    int vocab0;           // lm_head: first vocabulary row of this rank's slice
    int xf_off;           // float offset of the row-exchange flags in every buffer
};

__device__ __forceinline__ float* tp_slot(float* buf, const TpArgs& t, unsigned epoch) {
    return buf + kTpSlots + (size_t)(epoch & 1u) * t.world * t.ld;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Row-parallel exchange n, arrival (thread 0, after the CTA's pushes and a
// __syncthreads): the CTA's writes are ordered at system scope, then its flag
// slot on every rank is set to n.  One writer per slot: where every CTA of
// every rank added 1 to one counter per rank, world x grid atomics met on one
// address per exchange; these flag stores do not queue behind each other.
__device__ __forceinline__ void tp_flag_arrive(const TpArgs& t, unsigned n) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < t.world; ++r)
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(
                         reinterpret_cast<unsigned*>(t.peer[r] + t.xf_off) + t.rank * kTpMaxGrid + blockIdx.x),
                     "r"(n)
                     : "memory");
}

// Row-parallel exchange n, wait (warp 0 of every CTA): until every CTA of every
// rank has set its flag slot here to n; each lane watches every 32nd slot.
// Bounded like every wait (on a timeout the abort latch and the timeout bit
// are raised); returns the same answer on every lane.
__device__ __forceinline__ bool tp_flag_wait(const TpArgs& t, unsigned n, int G, unsigned* abort_flag,
                                             unsigned* status) {
    const int lane = threadIdx.x & 31;
    const unsigned* f = reinterpret_cast<const unsigned*>(t.peer[t.rank] + t.xf_off);
    const long long t0 = clock64();
    bool ok = true;
    unsigned it = 0;
    for (int r = 0; r < t.world && ok; ++r) {
        for (int c = lane; c < G && ok; c += 32) {
            while ((int)(ld_acquire_sys(f + r * kTpMaxGrid + c) - n) < 0) {
                if ((++it & 31u) != 0) continue;
                if (*reinterpret_cast<volatile unsigned*>(abort_flag)) {
                    ok = false;
                    break;
                }
                if (clock64() - t0 > kSpinLimitCycles) {
                    atomicOr(abort_flag, 1u);
                    atomicOr(status, kStatusTimeout);
                    ok = false;
                    break;
                }
            }
        }
    }
    return __all_sync(0xffffffffu, ok);
}

// Tell every rank that this rank's writes for argmax exchange `epoch` are done
// (one thread): one system-scope fence orders them before the flag stores
// (with the relaxed stores, a release pattern), which then go to every rank
// without waiting for each other (a release store per rank waited for the
// previous rank's store to be acknowledged over NVLink).
__device__ __forceinline__ void tp_signal(const TpArgs& t, unsigned epoch) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < t.world; ++r)
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(reinterpret_cast<unsigned*>(t.peer[r] + kTpFlags) +
                                                               t.rank),
                     "r"(epoch)
                     : "memory");
}

// Wait (one thread, bounded by about a second) until every rank has signalled
// `epoch`; gives up early when this launch aborts.  On a timeout it raises the
// abort latch and the timeout status bit.
__device__ __forceinline__ bool tp_wait(const TpArgs& t, unsigned epoch, unsigned* abort_flag,
                                        unsigned* status) {
    const unsigned* f = reinterpret_cast<const unsigned*>(t.peer[t.rank] + kTpFlags);
    const long long t0 = clock64();
    for (int r = 0; r < t.world; ++r) {
        while ((int)(ld_acquire_sys(f + r) - epoch) < 0) {
            if (*reinterpret_cast<volatile unsigned*>(abort_flag)) return false;
            if (clock64() - t0 > kSpinLimitCycles) {
                atomicOr(abort_flag, 1u);
                atomicOr(status, kStatusTimeout);
                return false;
            }
        }
    }
    return true;
}

struct GemvArgs {
    const void* w[3];
    const float* row_scale[3];  // TVB_I8_ROW scales or nullptr
    float tscale[3];            // per-tensor scale (1 for F16)
    int N;                      // rows per matrix (PLAIN/RESID/LMHEAD/GATEUP)
    int K;
    const float* x;             // input vector (unused when gathering the embedding)
    const uint16_t* embd;       // GM_QKV layer 0: gather x = f32(embd[token])
    float* x_out;               // GM_QKV layer 0: residual stream initialised from the gather
    const float* norm_w;        // prologue RMSNorm weight, nullptr = no norm
    float eps;
    float* y;                   // PLAIN: y; RESID: residual (in/out); GATEUP: h; LMHEAD: logits
    int nh, nkv, hd;            // GM_QKV geometry
    float* q_out;
    float* kcache;              // this layer's K rows [max_seq][Hk]
    float* vcache;
    const float* rope_cos;      // [max_seq][hd/2]
    const float* rope_sin;
    StepState* st;
    unsigned* status;
    int gather_token;           // GM_QKV: 1 on layer 0
    const float* attn_part;     // GM_RESID after attention: input = merge of these partials
    int attn_nsplit;            // splits per head in attn_part ([nh][nsplit][hd + 4])
    TpArgs tp;                  // world == 1: no tensor parallelism
};

__device__ __forceinline__ unsigned long long argmax_pack(float v, int idx) {
    uint32_t b = __float_as_uint(v);
    uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_index(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}
__device__ __forceinline__ float argmax_value(unsigned long long key) {
    uint32_t ord = (uint32_t)(key >> 32);
    uint32_t b = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
    return __uint_as_float(b);
}

// Row i of group g -> (matrix, row within matrix, valid).
template <int MODE, int R>
__device__ __forceinline__ bool group_row(const GemvArgs& a, int g, int i, int& m, int& row) {
    if (MODE == GM_QKV) {
        const int half = a.hd >> 1;
        int p = g;
        const int nq = a.nh * half, nk = a.nkv * half;
        if (p < nq) m = 0;
        else if (p < nq + nk) { m = 1; p -= nq; }
        else { m = 2; p -= nq + nk; }
        row = (p / half) * a.hd + (p % half) + i * half;
        return true;
    } else if (MODE == GM_GATEUP) {
        m = i;
        row = g;
        return row < a.N;
    } else {
        m = 0;
        row = g * R + i;
        return row < a.N;
    }
}

template <int MODE>
__host__ __device__ inline int gemv_units(const GemvArgs& a, int R) {
    if (MODE == GM_QKV) return (a.nh + 2 * a.nkv) * (a.hd >> 1);
    if (MODE == GM_GATEUP) return a.N;
    return (a.N + R - 1) / R;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    const uint64_t ua = (uint64_t)__float_as_uint(a.x) | ((uint64_t)__float_as_uint(a.y) << 32);
    const uint64_t ub = (uint64_t)__float_as_uint(b.x) | ((uint64_t)__float_as_uint(b.y) << 32);
    const uint64_t uc = (uint64_t)__float_as_uint(c.x) | ((uint64_t)__float_as_uint(c.y) << 32);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(ua), "l"(ub), "l"(uc));
    return make_float2(__uint_as_float((uint32_t)d), __uint_as_float((uint32_t)(d >> 32)));
}

// acc (two F32 lanes) += 8 weights . 8 activations, packed F32x2 FMAs.
__device__ __forceinline__ float2 dot8_h(uint4 u, const float4& xlo, const float4& xhi, float2 acc) {
    float w[8];
    h8_to_f8(u, w);
    acc = ffma2(make_float2(w[0], w[1]), make_float2(xlo.x, xlo.y), acc);
    acc = ffma2(make_float2(w[2], w[3]), make_float2(xlo.z, xlo.w), acc);
    acc = ffma2(make_float2(w[4], w[5]), make_float2(xhi.x, xhi.y), acc);
    acc = ffma2(make_float2(w[6], w[7]), make_float2(xhi.z, xhi.w), acc);
    return acc;
}
// (v.x, v.y, v.z, v.w) rotated left by r words.
__device__ __forceinline__ uint4 rot_words(const uint4& v, int r) {
    const uint4 t = (r & 1) ? make_uint4(v.y, v.z, v.w, v.x) : v;
    return (r & 2) ? make_uint4(t.z, t.w, t.x, t.y) : t;
}

// acc += 4 int8 weights . 4 activations.  Each biased byte (b + 128) is
// placed by one byte permute into the low mantissa of 2^23 (the float
// 2^23 + 128 + b); one packed add per pair removes 2^23 + 128 exactly.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ float2 dot4_i8(uint32_t u, const float4& x, float2 acc) {
    const uint32_t b = u ^ 0x80808080u;
    constexpr uint32_t kMagic = 0x4B000000u;   // bytes 4-7 of the permute: 00 00 00 4B
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    const float2 one = make_float2(1.0f, 1.0f);
    const float2 w01 = ffma2(make_float2(__uint_as_float(prmt(b, kMagic, 0x7540u)), __uint_as_float(prmt(b, kMagic, 0x7541u))),
                             one, bias);
    const float2 w23 = ffma2(make_float2(__uint_as_float(prmt(b, kMagic, 0x7542u)), __uint_as_float(prmt(b, kMagic, 0x7543u))),
                             one, bias);
    acc = ffma2(w01, make_float2(x.x, x.y), acc);
    acc = ffma2(w23, make_float2(x.z, x.w), acc);
    return acc;
}

// Shared memory layout (bytes):
//   [0, 1024)       reserved (phase descriptors, step scalars)
//   [1024, ..)      activation vector, K floats
//   [.., ..)        norm weight, K floats (staged before the inputs are ready)
//   [.., ..)        per-(chunk, row) partial sums of this CTA, nc * rows_cap floats
//   [.., ..)        epilogue operands: row scale and residual per local row
//                   (2 * rows_cap floats), RoPE cos/sin at this position
constexpr int kChunkBytes = 2048;   // one item: 4 x 512 B warp requests
// An item covers kChunkCols columns: one F16 row (2 KB), or two INT8 rows
// (1 KB each) multiplied with the same activations, so that every 16 bytes of
// INT8 weights cost the same 32 bytes of shared-memory activation reads as 16
// bytes of F16 weights (one INT8 row per item read 64: the shared-memory pipe,
// not HBM, bounded the INT8 rows).
constexpr int kChunkCols = 1024;
template <int WT>
__host__ __device__ constexpr int rows_per_item() { return WT == WT_F16 ? 1 : 2; }
constexpr int kDepth = 3;           // items in flight per warp

struct GemvSmem {
    int x_off, nw_off, part_off, pre_off, total;
};
constexpr int kMaxRopeHalf = 128;
__host__ __device__ inline GemvSmem gemv_smem_layout(int K, int esz, int rows_cap) {
    GemvSmem s;
    (void)esz;
    const int nc = (K + kChunkCols - 1) / kChunkCols;
    s.x_off = 1024;
    s.nw_off = s.x_off + ((K * 4 + 127) / 128) * 128;
    s.part_off = s.nw_off + ((K * 4 + 127) / 128) * 128;
    s.pre_off = s.part_off + ((nc * rows_cap * 4 + 127) / 128) * 128;
    s.total = s.pre_off + (((2 * rows_cap + 2 * kMaxRopeHalf) * 4 + 127) / 128) * 128;
    return s;
}
__host__ __device__ inline int gemv_rows_cap(int n_units, int grid, int R) {
    return ((n_units + grid - 1) / grid) * R;
}

// Geometry of one GEMV phase for this CTA/warp: the CTA's units [U0, U1)
// become local rows [0, nrows); items t = lgrp * nc + c, lgrp a group of
// rows_per_item local rows (row-major, so a warp's items are one contiguous
// span of the weight matrix for F16) are split evenly over the warps, this
// warp owning [t0, t0 + mine).
struct GemvGeo {
    int U0, U1, nrows, t0, mine, nc, rows_cap;
};

template <int MODE, int WT, int R>
__device__ __forceinline__ GemvGeo gemv_geo(const GemvArgs& a, int G, int b, int warp) {
    GemvGeo g;
    const int esz = (WT == WT_F16) ? 2 : 1;
    const int n_units = gemv_units<MODE>(a, R);
    (void)esz;
    g.nc = (a.K + kChunkCols - 1) / kChunkCols;
    g.rows_cap = gemv_rows_cap(n_units, G, R);
    g.U0 = (int)((long long)n_units * b / G);
    g.U1 = (int)((long long)n_units * (b + 1) / G);
    g.nrows = (g.U1 - g.U0) * R;
    constexpr int rpi = rows_per_item<WT>();
    const int items = ((g.nrows + rpi - 1) / rpi) * g.nc;
    g.t0 = (int)((long long)items * warp / kGemvWarps);
    g.mine = (int)((long long)items * (warp + 1) / kGemvWarps) - g.t0;
    return g;
}

// A warp's chunks in flight: slot j holds this lane's four 16-byte pieces.
struct ChunkBuf {
    uint4 v[kDepth][4];
};

// Request item k of this warp into slot j (all lanes; out-of-range -> zeros).
// F16: the item's 2 KB of one row as 4 x 512 B.  INT8: 1 KB of each of the
// item's two rows, [0, 2) the first row and [2, 4) the second.
template <int MODE, int WT, int R>
__device__ __forceinline__ void gemv_load(const GemvArgs& a, const GemvGeo& g, int k, uint4 (&dst)[4]) {
    const int esz = (WT == WT_F16) ? 2 : 1;
    constexpr int rpi = rows_per_item<WT>();
    const int row_bytes = a.K * esz;
    const int lane = threadIdx.x & 31;
    int bytes[rpi] = {};
    const unsigned char* src[rpi] = {};
    if (k < g.mine) {
        const int t = g.t0 + k;
        const int lg = t / g.nc, c = t - lg * g.nc;
#pragma unroll
        for (int q = 0; q < rpi; ++q) {
            const int lrow = lg * rpi + q;
            int m, row;
            if (lrow < g.nrows && group_row<MODE, R>(a, g.U0 + lrow / R, lrow % R, m, row)) {
                const int off = c * kChunkCols * esz;
                bytes[q] = min(kChunkCols * esz, row_bytes - off);
                src[q] = static_cast<const unsigned char*>(a.w[m]) + (size_t)row * row_bytes + off;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = (rpi == 1) ? 0 : (i >> 1);
        const int o = 512 * (rpi == 1 ? i : (i & 1)) + lane * 16;
        dst[i] = (o < bytes[q]) ? ld_stream16(src[q] + o) : make_uint4(0u, 0u, 0u, 0u);
    }
}

// Request this warp's first kDepth items of a phase (no dependence on inputs).
template <int MODE, int WT, int R>
__device__ __forceinline__ void gemv_prefetch(const GemvArgs& a, int G, int b, int warp, ChunkBuf& buf) {
    const GemvGeo g = gemv_geo<MODE, WT, R>(a, G, b, warp);
#pragma unroll
    for (int j = 0; j < kDepth; ++j) gemv_load<MODE, WT, R>(a, g, j, buf.v[j]);
}

struct GemvArgmax {
    float v;
    int i;
};

// Stage the phase's input-independent operands into shared memory: the norm
// weight, per-row output scales and the RoPE factors of this position.  Runs
// before the wait for the phase's inputs, so its loads overlap that wait.
// Warp 0 takes no part: its thread 0 polls the grid barrier, and a poll that
// started only after this thread's staging loads returned (they queue behind
// the weight prefetch) measured 30 us per 2B step slower.
template <int MODE, int WT, int R>
__device__ __forceinline__ void gemv_stage(const GemvArgs& a, unsigned char* smem, int G, int pos) {
    const int tid = threadIdx.x, warp = tid >> 5;
    const int esz = (WT == WT_F16) ? 2 : 1;
    const GemvGeo g = gemv_geo<MODE, WT, R>(a, G, blockIdx.x, warp);
    const GemvSmem L = gemv_smem_layout(a.K, esz, g.rows_cap);
    if (a.norm_w) {
        const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
        float4* nw4 = reinterpret_cast<float4*>(smem + L.nw_off);
        if (tid >= 32)
            for (int k4 = tid - 32; k4 < (a.K >> 2); k4 += kGemvThreads - 32) nw4[k4] = __ldg(w4 + k4);
    }
    float* pre_scale = reinterpret_cast<float*>(smem + L.pre_off);
    float* pre_res = pre_scale + g.rows_cap;
    for (int lr = tid - 32; tid >= 32 && lr < g.nrows; lr += kGemvThreads - 32) {
        int m, row;
        float sc = 1.0f;
        const bool v = group_row<MODE, R>(a, g.U0 + lr / R, lr % R, m, row);
        if (v) sc = a.row_scale[m] ? __ldg(a.row_scale[m] + row) : a.tscale[m];
        pre_scale[lr] = sc;
        // The residual a RESID phase adds to was last written two phases
        // earlier (o_proj: the previous layer's down or the layer-0 gather;
        // down: o_proj), with a grid barrier in between, so it can be staged
        // before the wait for this phase's inputs.  (Under tensor parallelism
        // the residual is folded by the next phase instead.)
        if (MODE == GM_RESID && !(a.tp.world > 1 && a.tp.index >= 0)) pre_res[lr] = v ? __ldcg(a.y + row) : 0.f;
    }
    if (MODE == GM_QKV) {
        float* pre_cos = pre_scale + 2 * g.rows_cap;
        float* pre_sin = pre_cos + kMaxRopeHalf;
        const int half = a.hd >> 1;
        for (int d = tid - 32; tid >= 32 && d < half; d += kGemvThreads - 32) {
            pre_cos[d] = __ldg(a.rope_cos + (size_t)pos * half + d);
            pre_sin[d] = __ldg(a.rope_sin + (size_t)pos * half + d);
        }
    }
}

// One GEMV phase whose constants are staged (gemv_stage), whose first kDepth
// items are already requested in `buf`, and whose inputs are ready: residual
// operands, activation prologue, chunk stream, epilogue.
// TP: the tensor-parallel decode kernel's instantiation (folds and pushes of
// partial rows); the single-GPU kernels compile those paths out.
// push0: row-parallel exchanges completed before this launch (slot parity).
template <int MODE, int WT, int R, bool TP = false>
__device__ __forceinline__ void gemv_run(const GemvArgs& a, unsigned char* smem, int G, int pos, int token,
                                         ChunkBuf& buf, GemvArgmax& best, unsigned push0 = 0) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, b = blockIdx.x;
    const int K = a.K;
    const int esz = (WT == WT_F16) ? 2 : 1;
    const GemvGeo g = gemv_geo<MODE, WT, R>(a, G, b, warp);
    const GemvSmem L = gemv_smem_layout(K, esz, g.rows_cap);
    float* xs = reinterpret_cast<float*>(smem + L.x_off);
    const float* nws = reinterpret_cast<const float*>(smem + L.nw_off);
    float* part = reinterpret_cast<float*>(smem + L.part_off);       // [c][lrow]
    float* pre_scale = reinterpret_cast<float*>(smem + L.pre_off);   // [lrow]
    float* pre_res = pre_scale + g.rows_cap;                         // [lrow]
    float* pre_cos = pre_res + g.rows_cap;                           // [hd/2]
    float* pre_sin = pre_cos + kMaxRopeHalf;

    // ---- residual operands (written by earlier phases) ---------------------------
    // row-parallel shard (o_proj, down): partial rows to every rank.  The
    // lm_head phase also carries an exchange index (its argmax), but no rows.
    const bool push = TP && MODE == GM_RESID && a.tp.world > 1 && a.tp.index >= 0;
    // (RESID: the residual operands were staged by gemv_stage)

    // ---- prologue: activation vector into shared memory ------------------------
    // One vectorised pass stores x*w and accumulates sum(x^2); 1/rms is applied
    // to the dot products in the epilogue, (W.(x*w))*inv, which keeps the
    // reduction off the critical path.  Activations are read through L2
    // (ld.global.cg): another CTA or kernel wrote them.
    __shared__ float red_ss[kGemvWarps];
    // tensor parallelism: the input is the residual plus the partial outputs of
    // every rank (summed in rank order, so every rank holds the same vector),
    // scaled by the sub-norm factor from the ranks' partial sums of squares
    const bool fold = TP && a.tp.world > 1 && a.tp.fold >= 0;
    const float* tp_in = nullptr;
    float tp_inv = 1.0f;
    if (fold) {
        tp_in = tp_slot(a.tp.peer[a.tp.rank], a.tp, push0 + (unsigned)a.tp.fold + 1u);
        float ss_all = 0.f;
        for (int r = 0; r < a.tp.world; ++r) ss_all += __ldcg(tp_in + (size_t)r * a.tp.ld + K);
        // tensor.cpp:672-673 over the full sub-norm length (norm_n == 0: no sub-norm)
        if (a.tp.norm_n > 0)
            tp_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss_all, (float)a.tp.norm_n), a.eps)));
    }
    {
        const uint16_t* esrc = nullptr;
        if (MODE == GM_QKV && a.gather_token) esrc = a.embd + (size_t)token * K;
        const float4* x4 = reinterpret_cast<const float4*>(a.x);
        const float4* w4 = a.norm_w ? reinterpret_cast<const float4*>(nws) : nullptr;
        float4* xs4 = reinterpret_cast<float4*>(xs);
        const int K4 = K >> 2;
        float ss = 0.f;
#pragma unroll 4
        for (int k4 = tid; k4 < K4; k4 += kGemvThreads) {
            float4 v;
            if (esrc) {
                const uint2 h = __ldg(reinterpret_cast<const uint2*>(esrc) + k4);
                const float2 l0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                const float2 l1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                v = make_float4(l0.x, l0.y, l1.x, l1.y);
                if (b == 0) reinterpret_cast<float4*>(a.x_out)[k4] = v;
            } else if (MODE == GM_RESID && a.attn_part) {
                // attention output = softmax-weighted merge of the per-split partials
                // (online-softmax rescaling, as in flash decoding)
                // all split loads are issued together (fixed trip count, predicated)
                const int hd = a.hd, h = (k4 * 4) / hd, d = (k4 * 4) - h * hd;
                const float* pb = a.attn_part + (size_t)h * a.attn_nsplit * (hd + 4);
                float ms[kMaxAttnSplits], ls[kMaxAttnSplits];
                float4 pv[kMaxAttnSplits];
#pragma unroll
                for (int sp = 0; sp < kMaxAttnSplits; ++sp) {
                    if (sp < a.attn_nsplit) {
                        const float* ps = pb + sp * (hd + 4);
                        ms[sp] = __ldcg(ps + hd);
                        ls[sp] = __ldcg(ps + hd + 1);
                        pv[sp] = __ldcg(reinterpret_cast<const float4*>(ps + d));
                    } else {
                        ms[sp] = -INFINITY;
                        ls[sp] = 0.f;
                        pv[sp] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
                float M = -INFINITY;
#pragma unroll
                for (int sp = 0; sp < kMaxAttnSplits; ++sp) M = fmaxf(M, ms[sp]);
                float Ls = 0.f;
                float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int sp = 0; sp < kMaxAttnSplits; ++sp) {
                    const float w = (ms[sp] == -INFINITY) ? 0.f : expf(ms[sp] - M);
                    Ls = fmaf(ls[sp], w, Ls);
                    o = make_float4(fmaf(pv[sp].x, w, o.x), fmaf(pv[sp].y, w, o.y), fmaf(pv[sp].z, w, o.z),
                                    fmaf(pv[sp].w, w, o.w));
                }
                const float inv = 1.0f / Ls;
                v = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
            } else if (fold) {
                v = __ldcg(x4 + k4);
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int r = 0; r < a.tp.world; ++r) {
                    const float4 p = __ldcg(reinterpret_cast<const float4*>(tp_in + (size_t)r * a.tp.ld) + k4);
                    acc = make_float4(acc.x + p.x, acc.y + p.y, acc.z + p.z, acc.w + p.w);
                }
                v = make_float4(__fadd_rn(v.x, acc.x * tp_inv), __fadd_rn(v.y, acc.y * tp_inv),
                                __fadd_rn(v.z, acc.z * tp_inv), __fadd_rn(v.w, acc.w * tp_inv));
                if (k4 % G == b) reinterpret_cast<float4*>(a.tp.x_out)[k4] = v;
            } else {
                v = __ldcg(x4 + k4);
            }
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            if (w4) {
                const float4 w = w4[k4];
                v = make_float4(v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w);
            }
            xs4[k4] = v;
        }
        ss = warp_sum(ss);
        if (lane == 0) red_ss[warp] = ss;
    }
    __syncthreads();
    trace_stamp(1);

    // ---- main loop: kDepth chunks in flight per warp ---------------------------------
    const int hsel = (lane >> 2) & 1;   // bank-conflict-free order for the F16 x loads
    const int qrot = (lane >> 1) & 3;   // and for the INT8 ones
    for (int k0 = 0; k0 < g.mine; k0 += kDepth) {
#pragma unroll
        for (int j = 0; j < kDepth; ++j) {
            const int k = k0 + j;
            if (k >= g.mine) break;
            const int t = g.t0 + k;
            const int lg = t / g.nc, c = t - lg * g.nc;
            const int e0 = c * kChunkCols;   // first column of the chunk
            float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0;
            float2 accB0 = acc0, accB1 = acc0;   // INT8: the item's second row
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (WT == WT_F16) {
                    const int e = e0 + 256 * i + lane * 8;
                    if (e < K) {
                        const float* xp = xs + e;
                        const float4 p0 = *reinterpret_cast<const float4*>(xp + 4 * hsel);
                        const float4 p1 = *reinterpret_cast<const float4*>(xp + 4 * (1 - hsel));
                        if (i & 1) acc1 = dot8_h(buf.v[j][i], hsel ? p1 : p0, hsel ? p0 : p1, acc1);
                        else acc0 = dot8_h(buf.v[j][i], hsel ? p1 : p0, hsel ? p0 : p1, acc0);
                    }
                } else if (i < 2) {
                    const int e = e0 + 512 * i + lane * 16;
                    if (e < K) {
                        // the lane's 16 activations as 4 float4, read in a rotated
                        // order (quad (q + lane / 2) % 4): conflict-free shared memory;
                        // each is used by both rows of the item
                        const float4* xp = reinterpret_cast<const float4*>(xs + e);
                        const float4 x0 = xp[qrot], x1 = xp[(qrot + 1) & 3], x2 = xp[(qrot + 2) & 3],
                                     x3 = xp[(qrot + 3) & 3];
                        const uint4 w = rot_words(buf.v[j][i], qrot);
                        acc0 = dot4_i8(w.x, x0, acc0);
                        acc1 = dot4_i8(w.y, x1, acc1);
                        acc0 = dot4_i8(w.z, x2, acc0);
                        acc1 = dot4_i8(w.w, x3, acc1);
                        const uint4 u = rot_words(buf.v[j][i + 2], qrot);
                        accB0 = dot4_i8(u.x, x0, accB0);
                        accB1 = dot4_i8(u.y, x1, accB1);
                        accB0 = dot4_i8(u.z, x2, accB0);
                        accB1 = dot4_i8(u.w, x3, accB1);
                    }
                }
            }
            // refill this slot with the item kDepth ahead
            gemv_load<MODE, WT, R>(a, g, k + kDepth, buf.v[j]);
            const float v = warp_sum((acc0.x + acc0.y) + (acc1.x + acc1.y));
            constexpr int rpi = rows_per_item<WT>();
            if (lane == 0) part[c * g.rows_cap + lg * rpi] = v;
            if (rpi == 2) {
                const float vb = warp_sum((accB0.x + accB0.y) + (accB1.x + accB1.y));
                if (lane == 0 && lg * rpi + 1 < g.nrows) part[c * g.rows_cap + lg * rpi + 1] = vb;
            }
        }
    }
    __syncthreads();
    trace_stamp(2);

    // tensor.cpp:675-676: rms = sqrt(ss/n + eps); inv = 1/rms
    float inv = 1.0f, ss_local = 0.f;
    size_t tp_off = 0;   // push: offset of this rank's partial rows in every rank's buffer
    if (a.norm_w) {
        for (int w = 0; w < kGemvWarps; ++w) ss_local += red_ss[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss_local, (float)K), a.eps)));
    }
    if (push) {
        // the sub-norm factor needs every rank's sum of squares: apply it when folding
        inv = 1.0f;
        const unsigned e = push0 + (unsigned)a.tp.index + 1u;
        tp_off = (size_t)(tp_slot(a.tp.peer[0], a.tp, e) - a.tp.peer[0]) + (size_t)a.tp.rank * a.tp.ld;
        if (b == 0 && tid == 0)
            for (int r = 0; r < a.tp.world; ++r) a.tp.peer[r][tp_off + a.N] = ss_local;
    }

    // ---- epilogue: one thread per unit -----------------------------------------------
    for (int lu = tid; lu < g.U1 - g.U0; lu += kGemvThreads) {
        const int gu = g.U0 + lu;
        float y[R];
        int ms[R], rows[R];
        bool valid[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float t = 0.f;
            for (int c = 0; c < g.nc; ++c) t += part[c * g.rows_cap + lu * R + r];
            valid[r] = group_row<MODE, R>(a, gu, r, ms[r], rows[r]);
            const float sc = pre_scale[lu * R + r] * inv;
            y[r] = (sc == 1.0f) ? t : t * sc;
        }
        if (MODE == GM_GATEUP) {
            // relu2_d then mul_d (ops_cuda.cu:123-130, 116-121)
            const float gr = fmaxf(y[0], 0.0f);
            a.y[rows[0]] = __fmul_rn(__fmul_rn(gr, gr), y[1]);
        } else if (MODE == GM_QKV) {
            const int half = a.hd >> 1;
            const int d = rows[0] % a.hd;   // < half
            const int head = rows[0] / a.hd;
            float y0 = y[0], y1 = y[1];
            if (ms[0] < 2) {
                // NeoX pair (d, d + hd/2), tensor.cpp:918-925
                const float cs = pre_cos[d];
                const float sn = pre_sin[d];
                const float r0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                const float r1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
                y0 = r0;
                y1 = r1;
            }
            if (ms[0] == 0) {
                a.q_out[head * a.hd + d] = y0;
                a.q_out[head * a.hd + d + half] = y1;
            } else {
                float* dst = (ms[0] == 1 ? a.kcache : a.vcache) + (size_t)pos * a.nkv * a.hd +
                             head * a.hd + d;
                dst[0] = y0;
                dst[half] = y1;
            }
        } else {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (!valid[r]) continue;
                if (MODE == GM_PLAIN) a.y[rows[r]] = y[r];
                else if (MODE == GM_RESID) {
                    if (push) {
                        pre_res[lu * R + r] = y[r];   // pushed below, 16 bytes at a time
                    } else {
                        a.y[rows[r]] = __fadd_rn(pre_res[lu * R + r], y[r]);
                    }
                } else {
                    a.y[rows[r]] = y[r];
                    if (y[r] > best.v) { best.v = y[r]; best.i = rows[r] + a.tp.vocab0; }
                }
            }
        }
    }
    if (push) {
        // The CTA's rows [U0, U1) (R == 1: one row per unit) to every rank's
        // slot: 16-byte stores for the aligned middle, single floats at the edges
        // (slot offsets and ld are multiples of 4 floats).
        __syncthreads();
        const int r0 = g.U0, r1 = g.U1;
        const int a0 = min(r1, (r0 + 3) & ~3), a1 = max(a0, r1 & ~3);
        const int nv = (a1 - a0) >> 2, ne = (a0 - r0) + (r1 - a1);
        for (int i = tid; i < a.tp.world * (nv + ne); i += kGemvThreads) {
            const int q = i / (nv + ne), j = i - q * (nv + ne);
            float* dst = a.tp.peer[q] + tp_off;
            if (j < nv) {
                const int row = a0 + 4 * j;
                const float* v = pre_res + (row - r0);
                *reinterpret_cast<float4*>(dst + row) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
                const int e = j - nv;
                const int row = e < a0 - r0 ? r0 + e : a1 + (e - (a0 - r0));
                dst[row] = pre_res[row - r0];
            }
        }
    }
    trace_stamp(3);
}

// LM-head completion: CTA-wide argmax, global max, and -- in the last CTA to
// finish -- publication of the step's token and advance of the step state.
template <bool TP = false>
__device__ __forceinline__ void lmhead_finish(const GemvArgs& a, const GemvArgmax& best, unsigned epoch0 = 0) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ unsigned long long kbest[kGemvWarps];
    unsigned long long key = (best.v == -INFINITY) ? 0ull : argmax_pack(best.v, best.i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if (lane == 0) kbest[warp] = key;
    __syncthreads();
    if (tid == 0) {
        unsigned long long k = 0;
        for (int w = 0; w < kGemvWarps; ++w) k = kbest[w] > k ? kbest[w] : k;
        if (k) atomicMax(&a.st->argmax_key, k);
        __threadfence();
        const unsigned done = atomicAdd(&a.st->lm_done, 1u);
        if (done == gridDim.x - 1) {
            // Last CTA: publish this step's argmax and advance the step state.
            __threadfence();
            unsigned long long fin = atomicAdd(&a.st->argmax_key, 0ull);
            if (TP && a.tp.world > 1) {
                // vocabulary-parallel lm_head: the step's token is the largest
                // key over the ranks' slices (every rank takes the same one)
                const unsigned e = epoch0 + (unsigned)a.tp.index + 1u;
                for (int r = 0; r < a.tp.world; ++r)
                    reinterpret_cast<unsigned long long*>(a.tp.peer[r] + kTpKeys)[a.tp.rank] = fin;
                tp_signal(a.tp, e);
                if (tp_wait(a.tp, e, &a.st->abort, &a.st->status)) {
                    const unsigned long long* keys =
                        reinterpret_cast<const unsigned long long*>(a.tp.peer[a.tp.rank] + kTpKeys);
                    for (int r = 0; r < a.tp.world; ++r) {
                        const unsigned long long k = __ldcg(keys + r);
                        fin = k > fin ? k : fin;
                    }
                    a.st->tp_epoch = e;   // (the decode step's exit writes the same value)
                }
            }
            // No key at all (every logit NaN): token 0, what a first-index
            // argmax that skips NaN (every comparison false) returns; never the
            // out-of-range index an empty key would decode to.
            const int tok = fin ? argmax_index(fin) : 0;
            a.st->next_token = tok;
            a.st->max_logit = fin ? argmax_value(fin) : -INFINITY;
            a.st->token = tok;
            a.st->pos = a.st->pos + 1;
            a.st->argmax_key = 0ull;
            a.st->lm_done = 0u;
        }
    }
}

// Stand-alone launch of one GEMV phase (the per-op API and tests).
template <int MODE, int WT, int R, bool TP = false>
__global__ void __launch_bounds__(kGemvThreads, 1)
stream_gemv_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
#ifdef TVB_PHASE_TRACE
    if (threadIdx.x == 0) s_trace_row = nullptr;   // stand-alone launches are not traced
#endif
    ChunkBuf buf;
    gemv_prefetch<MODE, WT, R>(a, gridDim.x, blockIdx.x, threadIdx.x >> 5, buf);
    pdl_launch_dependents();
    pdl_wait();
    const int pos = (MODE == GM_QKV) ? __ldcg(&a.st->pos) : 0;
    const int token = (MODE == GM_QKV && a.gather_token) ? __ldcg(&a.st->token) : 0;
    gemv_stage<MODE, WT, R>(a, smem, gridDim.x, pos);
    __syncthreads();   // the staged operands are read by other threads than staged them
    GemvArgmax best{-INFINITY, 0};
    gemv_run<MODE, WT, R, TP>(a, smem, gridDim.x, pos, token, buf, best);
    if (MODE == GM_LMHEAD) lmhead_finish<TP>(a, best, TP ? __ldcg(&a.st->tp_epoch) : 0u);
}

}  // namespace tvb
