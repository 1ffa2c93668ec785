// Batched prefill kernels for sm_100a (see prefill.h).
//
// pf_gemm_kernel: one CTA computes a 128-token x 256-weight-row tile of
// acc = X . W^T.  Warp roles: warp 0 lane 0 issues TMA loads into a 3-stage
// shared-memory ring (128B-swizzled, K-major tiles: the activation planes hi/lo
// [128 tokens][64 k] and the weight tile [256 rows][64 k], loaded as two
// 128-row halves so one tile can pair rows of different matrices: gate with
// up, q/k/v heads); warp 1 lane 0 issues tcgen05.mma (M=128, N=256, K=16,
// F16 x F16 -> F32 in TMEM) and frees each stage with tcgen05.commit; warp 2
// owns the TMEM allocation; warps 4-7 read the accumulator back with
// tcgen05.ld (warp w sees TMEM lanes 32*(w%4) .. +31 = its 32 tokens) and run
// the fused epilogue.  Every mbarrier wait is bounded: a stall of about a
// second sets the status word and the CTA leaves through the normal exit path
// (TMEM freed, outstanding TMA writes waited for).
//
// Activations reach the tensor cores as two F16 planes, x = (hi + lo) * 2^e
// with a power-of-two row exponent e chosen so the row's largest magnitude
// lies in [2^14, 2^15): hi carries 11 significant bits, lo the next 11, so
// (hi + lo) reproduces the F32 activations to about 2^-22 of the row's largest
// element and the products with exact F16 weights accumulate in F32, as the
// reference's F32 x F16 GEMV/GEMM does (cuda/ops_cuda.cu:46-71, 269-294).
#include "prefill.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "stream.cuh"
#include "tcgen05.cuh"

namespace tvb {

// ---------------------------------------------------------------------------
// GEMM kernel
// ---------------------------------------------------------------------------
constexpr int kPfBM = 128;                         // tokens per tile (MMA M, TMEM lanes)
constexpr int kPfBK = 64;                          // k per stage: 128 B of F16 = one swizzle row
constexpr int kPfStages = 3;
constexpr int kPfThreads = 256;
constexpr int kPfPlane = kPfBM * kPfBK * 2;        // 16 KB activation plane per stage
constexpr int kPfHalf = 128 * kPfBK * 2;           // 16 KB weight half-tile per stage
// NH = 128-row weight halves per tile (2: 256 rows, the default; 1: 128 rows
// for projections with too few 256-row tiles to cover the SMs)
__host__ __device__ constexpr int pf_stage_bytes(int nh) { return 2 * kPfPlane + nh * kPfHalf; }
// after the stage ring: 1 KB of barriers, then two 4 KB output stages (32 x 32
// floats, 1024-byte aligned for the 128-byte swizzle) per epilogue warp
constexpr int kPfBarBytes = 1024;
constexpr int kPfOutStage = 32 * 32 * 4;
constexpr int kPfOutBytes = 4 * 2 * kPfOutStage;
__host__ __device__ constexpr int pf_smem_bytes(int nh) {
    return kPfStages * pf_stage_bytes(nh) + 1024 + kPfBarBytes + kPfOutBytes;
}

struct PfMaps {
    CUtensorMap xh, xl, w[3];
    // epilogue outputs (PfArgs::tma_out): STORE / RESID / GATEUP: out[0] over
    // y [S][rows0]; QKV: out[0..2] over q_out [S][nh * hd] and this layer's K / V
    // cache rows [pos0 + S][nkv * hd].  F32, 32 x 32 boxes, 128-byte swizzle.
    CUtensorMap out[3];
};

struct PfArgs {
    int mode, S, K, nk, use_lo;
    int rows[3];
    const float* row_scales[3];
    float scale[3];
    const int* row_exp;   // per token: activations are (hi + lo) * 2^row_exp
    float* y;
    int ldy;
    int nh, nkv, hd, pos0;
    float* q_out;
    float* kcache;
    float* vcache;
    const float* rope_cos;
    const float* rope_sin;
    const int* row_pos;      // per-row positions (rows are sequences), or nullptr
    size_t kv_slot_stride;   // per-row KV cache offset when row_pos is given
    unsigned* status;
    float* part;             // split-K: raw partials [ksplit][S][width]
    int ksplit, width;       // width = tiles * 128 * NH
    int w_static;            // no earlier kernel of the stream writes the weights
    // persistent stream-K kernel (pf_gemm_sk_kernel)
    int sk_total;            // k-block iterations of all tiles: units x nk
    int sk_mtiles;           // token tiles per weight tile (unit u: weight tile u / sk_mtiles)
    unsigned sk_epoch;       // value this launch writes into the flags of finished partial sums
    unsigned* sk_flags;      // [gridDim.x][4]: one per epilogue warp
    int tma_out;             // outputs leave through TMA stores (maps.out), else per-thread stores
};

// Position of activation row s, and the offset of its KV cache slot.
__device__ __forceinline__ int pf_pos(const PfArgs& a, int s) { return a.row_pos ? __ldg(a.row_pos + s) : a.pos0 + s; }
__device__ __forceinline__ size_t pf_slot(const PfArgs& a, int s) {
    return a.row_pos ? (size_t)s * a.kv_slot_stride : 0;
}

// Which matrix and first row feed half `h` (128 rows) of column tile `tile`
// (NH halves per tile).
__host__ __device__ inline bool pf_half(const PfArgs& a, int nh, int tile, int h, int& mi, int& row) {
    if (a.mode == PF_GATEUP) {
        mi = h;
        row = tile * 128;
        return row < a.rows[h];
    }
    if (a.mode == PF_QKV) {
        int slot = tile * nh + h;
        if (slot < a.nh) { mi = 0; row = slot * 128; return true; }
        slot -= a.nh;
        if (slot < a.nkv) { mi = 1; row = slot * 128; return true; }
        slot -= a.nkv;
        mi = 2;
        row = slot * 128;
        return slot < a.nkv;
    }
    mi = 0;
    row = tile * 128 * nh + h * 128;
    return row < a.rows[0];
}

__device__ __forceinline__ float pf_row_scale(const PfArgs& a, int mi, int n) {
    return a.row_scales[mi] ? __ldg(a.row_scales[mi] + n) : a.scale[mi];
}

// Store 32 consecutive values (vector stores when aligned), optionally adding
// to what is there; only the first `count` are written.
__device__ __forceinline__ void pf_store32(float* dst, const float (&v)[32], int count, bool add) {
    if (count >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            if (add) {
                const float4 p = d4[j];
                o = make_float4(__fadd_rn(p.x, o.x), __fadd_rn(p.y, o.y), __fadd_rn(p.z, o.z), __fadd_rn(p.w, o.w));
            }
            d4[j] = o;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < count) dst[j] = add ? __fadd_rn(dst[j], v[j]) : v[j];
    }
}

__device__ __forceinline__ void pf_fail(const PfArgs& a, volatile int* abort_flag) {
    *abort_flag = 1;
    if (a.status) atomicOr(a.status, kStatusTimeout);
}

// While the MMAs of a tile run, its epilogue warp asks L2 for the RoPE rows of
// its 32 positions (QKV), which later weight traffic has usually evicted.
template <int NH>
__device__ __forceinline__ void pf_epilogue_prefetch(const PfArgs& a, int s_base, int lane) {
    const int nrows = min(32, a.S - s_base);
    if (a.mode != PF_QKV || nrows <= 0) return;
    const int half = a.hd >> 1;
    for (int i = lane; i < 32 * 2; i += 32) {
        const int r = i >> 1;
        if (r >= nrows) continue;
        const size_t o = (size_t)pf_pos(a, s_base + r) * half + (i & 1) * 32;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.rope_cos + o));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.rope_sin + o));
    }
}

// This lane's row scale 2^row_exp (1 past the rows).
__device__ __forceinline__ float pf_e2(const PfArgs& a, int s) {
    return (s < a.S && a.row_exp) ? ldexpf(1.0f, a.row_exp[s]) : 1.0f;
}

// TMA stores of a 32 x 32 F32 box from shared memory (bulk async-groups).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}
// y[box] += box (F32 add, one rounding per element)
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most one group of this thread still reading shared memory
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every group of this thread complete (its writes performed)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Where the finished 32-column chunks of one warp's 32 token rows go.  TMA
// mode: the warp's rows are written into one of its two 128-byte-swizzled
// shared-memory boxes and lane 0 issues a tensor store (or reduce-add) of the
// 32 x 32 box; the tensor map clips rows past S and columns past the matrix.
// Otherwise: per-thread stores of the row (lanes past S store nothing).
struct PfEmit {
    const PfMaps* maps;
    uint32_t box[2];   // this warp's two stages (shared addresses)
    int nb;            // stage of the next box
    int lane;
    bool tma;
    bool srow;         // this lane's row exists

    // which: tensor map index; (x, y): box origin (column, row of the warp's
    // first row); dst / count / add: the per-thread fallback for this lane's row
    __device__ __forceinline__ void put(int which, int x, int y, bool add, float* dst, int count,
                                        const float (&v)[32]) {
        if (!tma) {
            if (srow) pf_store32(dst, v, count, add);
            return;
        }
        if (lane == 0) bulk_wait_read1();   // the box used two puts ago has been read
        __syncwarp();
        const uint32_t b = box[nb];
        nb ^= 1;
#pragma unroll
        for (int c = 0; c < 8; ++c)
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(b + sw128_offset(lane, c)), "f"(v[4 * c]),
                         "f"(v[4 * c + 1]), "f"(v[4 * c + 2]), "f"(v[4 * c + 3])
                         : "memory");
        fence_proxy_async_smem_cta();
        __syncwarp();
        if (lane == 0) {
            if (add) tma_reduce_add_2d(&maps->out[which], x, y, b);
            else tma_store_2d(&maps->out[which], x, y, b);
            bulk_commit();
        }
    }
    // before the stages are used otherwise, or the results are needed
    __device__ __forceinline__ void drain_reads() {
        if (tma && lane == 0) bulk_wait_read0();
        __syncwarp();
    }
    __device__ __forceinline__ void finish() {
        if (tma && lane == 0) bulk_wait_all();
        __syncwarp();
    }
};

// Epilogue of one 128-token x (128 * NH)-row tile for this thread's token row
// s (warp rows s_base .. s_base + 31): get(col, v) yields the row's sums of
// accumulator columns [col, col + 32) already scaled by the row's 2^row_exp
// (warp-collective: every lane calls it, in the same order); every finished
// 32-column chunk leaves through `out`.
template <int NH, class Get>
__device__ __forceinline__ void pf_tile_epilogue(const PfArgs& a, int s_base, int lane, const int (&mi)[2],
                                                 const int (&row)[2], const bool (&hv)[2], Get&& get, PfEmit& out) {
    const int s = s_base + lane;
    float v0[32], v1[32];
    if (a.mode == PF_GATEUP) {
        // relu2_d then mul_d (ops_cuda.cu:123-130, 116-121)
        for (int c = 0; c < 4; ++c) {
            __syncwarp();
            get(c * 32, v0);
            get(128 + c * 32, v1);
            const int n0 = row[0] + c * 32;
            if (!(hv[0] && hv[1]) || n0 >= a.rows[0]) continue;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int n = min(n0 + j, a.rows[0] - 1);
                const float g = __fmul_rn(v0[j], pf_row_scale(a, 0, n));
                const float u = __fmul_rn(v1[j], pf_row_scale(a, 1, n));
                const float gr = fmaxf(g, 0.0f);
                v0[j] = __fmul_rn(__fmul_rn(gr, gr), u);
            }
            out.put(0, n0, s_base, false, a.y + (size_t)s * a.ldy + n0, a.rows[0] - n0, v0);
        }
    } else if (a.mode == PF_QKV) {
        const int half = a.hd >> 1;   // 64
        const int pos = s < a.S ? pf_pos(a, s) : 0;
        for (int h = 0; h < NH; ++h) {
            const int head = row[h] / a.hd;
            for (int c = 0; c < 2; ++c) {
                __syncwarp();
                // RoPE factors of this row's position (2 x 128 contiguous bytes)
                float4 cs4[8], sn4[8];
                const bool rope = hv[h] && mi[h] < 2;
                if (rope) {
                    const float4* cp = reinterpret_cast<const float4*>(a.rope_cos + (size_t)pos * half + c * 32);
                    const float4* sp = reinterpret_cast<const float4*>(a.rope_sin + (size_t)pos * half + c * 32);
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        cs4[t] = __ldg(cp + t);
                        sn4[t] = __ldg(sp + t);
                    }
                }
                get(h * 128 + c * 32, v0);
                get(h * 128 + half + c * 32, v1);
                if (!hv[h]) continue;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int d = c * 32 + j;
                    float y0 = __fmul_rn(v0[j], pf_row_scale(a, mi[h], row[h] + d));
                    float y1 = __fmul_rn(v1[j], pf_row_scale(a, mi[h], row[h] + d + half));
                    if (rope) {
                        // NeoX pair (d, d + hd/2), tensor.cpp:918-925
                        const float4 c4 = cs4[j >> 2], s4 = sn4[j >> 2];
                        const float cs = (j & 3) == 0 ? c4.x : (j & 3) == 1 ? c4.y : (j & 3) == 2 ? c4.z : c4.w;
                        const float sn = (j & 3) == 0 ? s4.x : (j & 3) == 1 ? s4.y : (j & 3) == 2 ? s4.z : s4.w;
                        const float t0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                        const float t1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
                        y0 = t0;
                        y1 = t1;
                    }
                    v0[j] = y0;
                    v1[j] = y1;
                }
                float* dst;
                if (mi[h] == 0) dst = a.q_out + (size_t)s * a.nh * a.hd + head * a.hd;
                else
                    dst = (mi[h] == 1 ? a.kcache : a.vcache) + pf_slot(a, s) + (size_t)pos * a.nkv * a.hd +
                          head * a.hd;
                // q rows are token rows; K/V rows are positions pos0 + s
                const int y = mi[h] == 0 ? s_base : a.pos0 + s_base;
                out.put(mi[h], head * a.hd + c * 32, y, false, dst + c * 32, 32, v0);
                out.put(mi[h], head * a.hd + half + c * 32, y, false, dst + half + c * 32, 32, v1);
            }
        }
    } else {
        const bool add = a.mode == PF_RESID;
        for (int h = 0; h < NH; ++h) {
            for (int c = 0; c < 4; ++c) {
                __syncwarp();
                get(h * 128 + c * 32, v0);
                const int n0 = row[h] + c * 32;
                if (!hv[h] || n0 >= a.rows[0]) continue;
#pragma unroll
                for (int j = 0; j < 32; ++j) v0[j] = __fmul_rn(v0[j], pf_row_scale(a, 0, min(n0 + j, a.rows[0] - 1)));
                out.put(0, n0, s_base, add, a.y + (size_t)s * a.ldy + n0, a.rows[0] - n0, v0);
            }
        }
    }
}

template <int NH>
__global__ void __launch_bounds__(kPfThreads, 1)
pf_gemm_kernel(const __grid_constant__ PfMaps maps, const __grid_constant__ PfArgs a) {
    constexpr int kPfStage = pf_stage_bytes(NH);
    constexpr uint32_t kPfTmemCols = 128 * NH;
    extern __shared__ unsigned char pf_smem_raw[];
    const uint32_t raw = smem_u32(pf_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;   // 128B-swizzled tiles want 1024-B alignment
    unsigned char* smem = pf_smem_raw + (base - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPfStages * kPfStage);
    uint64_t* empty = full + kPfStages;
    uint64_t* done = empty + kPfStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued = const_cast<int*>(abort_flag) + 1;     // k-blocks requested by the producer
    int* consumed = issued + 1;                         // k-blocks the MMA warp saw land

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, s0 = blockIdx.y * kPfBM;
    // split-K: this CTA's k-blocks [kb0, kb0 + nkb)
    const int kb0 = (int)((long long)a.nk * blockIdx.z / gridDim.z);
    const int nkb = (int)((long long)a.nk * (blockIdx.z + 1) / gridDim.z) - kb0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kPfStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        *issued = 0;
        *consumed = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kPfTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();   // (programmatic launch) the activations come from the previous kernel
    pdl_launch_dependents();

    int mi[2], row[2];
    bool hv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) hv[h] = h < NH && pf_half(a, NH, tile, h, mi[h], row[h]);

    if (warp == 0 && lane == 0) {
        // ---- producer: TMA ring ------------------------------------------------------
        prefetch_tmap(&maps.xh);
        if (a.use_lo) prefetch_tmap(&maps.xl);
        const uint32_t bytes =
            (uint32_t)(kPfPlane * (a.use_lo ? 2 : 1) + (hv[0] ? kPfHalf : 0) + (hv[1] ? kPfHalf : 0));
        int i = 0;
        for (; i < nkb; ++i) {
            const int s = i % kPfStages, r = i / kPfStages, kx = (kb0 + i) * kPfBK;
            if (r > 0 && !mbar_wait_bounded(&empty[s], (uint32_t)((r - 1) & 1))) {
                pf_fail(a, abort_flag);
                break;
            }
            if (*abort_flag) break;
            const uint32_t st = base + (uint32_t)(s * kPfStage);
            mbar_expect_tx(&full[s], bytes);
            tma_load_2d(st, &maps.xh, kx, s0, &full[s]);
            if (a.use_lo) tma_load_2d(st + kPfPlane, &maps.xl, kx, s0, &full[s]);
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (hv[h]) tma_load_2d(st + 2 * kPfPlane + h * kPfHalf, &maps.w[mi[h]], kx, row[h], &full[s]);
        }
        *issued = i;
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----------------------------------------------------------------
        constexpr uint32_t idesc = umma_idesc_f16(kPfBM, 128 * NH);
        int kb = 0;
        for (; kb < nkb; ++kb) {
            const int s = kb % kPfStages, r = kb / kPfStages;
            if (!mbar_wait_bounded(&full[s], (uint32_t)(r & 1))) {
                pf_fail(a, abort_flag);
                break;
            }
            tc_fence_after();
            const uint32_t st = base + (uint32_t)(s * kPfStage);
#pragma unroll
            for (int kk = 0; kk < kPfBK / 16; ++kk) {
                const uint64_t bdesc = sw128_desc(st + 2 * kPfPlane + kk * 32);
                tc_mma(tmem, sw128_desc(st + kk * 32), bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
                if (a.use_lo) tc_mma(tmem, sw128_desc(st + kPfPlane + kk * 32), bdesc, idesc, 1u);
            }
            tc_commit(&empty[s]);   // stage s is free once these MMAs have read it
        }
        *consumed = kb;
        tc_commit(done);            // accumulator complete (or the MMAs issued so far)
    } else if (warp >= 4) {
        // ---- epilogue ------------------------------------------------------------------
        const int q = warp & 3;
        const int s = s0 + 32 * q + lane;
        const bool srow = s < a.S;
        if (gridDim.z == 1) pf_epilogue_prefetch<NH>(a, s0 + 32 * q, lane);
        const bool ok = mbar_wait_bounded(done, 0u);
        tc_fence_after();
        if (!ok) pf_fail(a, abort_flag);
        const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
        // accumulator columns [col, col + 32) of this thread's token row
        auto fetch = [&](int col, uint32_t (&r)[32]) {
            tmem_ld32(trow + col, r);
            tmem_wait_ld();
        };
        if (ok && !*abort_flag) {
            uint32_t r0[32];
            float v0[32];
            if (gridDim.z > 1) {
                // split-K: raw sums of this k range; pf_splitk_epilogue finishes
                float* dst = a.part + ((size_t)blockIdx.z * a.S + s) * a.width + (size_t)tile * 128 * NH;
                for (int c = 0; c < 4 * NH; ++c) {
                    __syncwarp();
                    fetch(c * 32, r0);
                    if (!srow) continue;
#pragma unroll
                    for (int j = 0; j < 32; ++j) v0[j] = __uint_as_float(r0[j]);
                    pf_store32(dst + c * 32, v0, 32, false);
                }
            } else {
                const uint32_t ob = base + (uint32_t)(kPfStages * kPfStage + kPfBarBytes + q * 2 * kPfOutStage);
                PfEmit out{&maps, {ob, ob + (uint32_t)kPfOutStage}, 0, lane, a.tma_out != 0, srow};
                const float e2 = pf_e2(a, s);
                pf_tile_epilogue<NH>(a, s0 + 32 * q, lane, mi, row, hv, [&](int col, float (&v)[32]) {
                    fetch(col, r0);
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r0[j]) * e2;
                }, out);
                out.finish();
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        // leave no TMA write in flight into this CTA's shared memory
        for (int kb = *consumed; kb < *issued; ++kb)
            mbar_wait_bounded(&full[kb % kPfStages], (uint32_t)((kb / kPfStages) & 1));
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// Persistent stream-K GEMM.  The U = weight tiles x token tiles output tiles
// ("units", unit u: weight tile u / mtiles, token tile u % mtiles), each nk
// k-blocks long, are laid end to end and CTA c of G takes the iterations
// [T c / G, T (c + 1) / G) of the T = U nk, so every SM gets the same number of
// k-blocks whatever U is.  A CTA's range is a run of segments (the part of one
// unit inside the range); the TMA producer and the MMA warp run through them
// without draining the stage ring, and the accumulator is double-buffered in
// TMEM (2 x 128 * NH columns), so the epilogue of one segment overlaps the
// MMAs of the next.  A unit cut by range boundaries is finished by its owner,
// the CTA holding its first k-block (always the last segment of the owner's
// range): every later CTA that holds a piece of it (its first segment) stores
// the piece's raw sums in its workspace slot part[c] ([128 tokens][128 * NH])
// and sets its flags (one per epilogue warp) to this launch's epoch; the owner
// waits for those flags, adds the pieces in k order to its own sums and runs
// the epilogue.  Pieces are computed first and owners wait last, so no CTA
// waits on one that is waiting; with at most one CTA per SM and G <= SMs all
// CTAs are resident together.  Every wait is bounded.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int sk_begin(const PfArgs& a, int c) {
    return (int)((long long)a.sk_total * c / gridDim.x);
}

struct PfSeg {
    int u, kb0, nkb;
    bool piece;   // starts inside its unit: raw sums go to this CTA's workspace slot
    int helpers;  // owner of a unit that later CTAs finish: how many hold pieces of it
};

__device__ __forceinline__ PfSeg pf_seg(const PfArgs& a, int it, int it1) {
    PfSeg g;
    g.u = it / a.nk;
    g.kb0 = it - g.u * a.nk;
    const int uend = (g.u + 1) * a.nk;
    const int end = min(it1, uend);
    g.nkb = end - it;
    g.piece = g.kb0 > 0;
    g.helpers = 0;
    if (!g.piece && end < uend)
        for (int c = blockIdx.x + 1; c < (int)gridDim.x && sk_begin(a, c) < uend; ++c) ++g.helpers;
    return g;
}

// Stream-K piece workspace: slot c (one per CTA) holds, per epilogue warp q and
// 32-column chunk, 8 float4 slices of the warp's 32 rows, lane-minor, so that
// writer (the piece's CTA) and reader (the owner) both move 512 contiguous
// bytes per instruction.  Float4 index of (slot, q, chunk, slice 0, lane).
__device__ __forceinline__ size_t pf_piece_idx(int slot, int q, int chunk, int W, int lane) {
    return ((((size_t)slot * 4 + q) * (W / 32) + chunk) * 8) * 32 + lane;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_u32_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <int NH>
__global__ void __launch_bounds__(kPfThreads, 1)
pf_gemm_sk_kernel(const __grid_constant__ PfMaps maps, const __grid_constant__ PfArgs a) {
    constexpr int kPfStage = pf_stage_bytes(NH);
    constexpr int W = 128 * NH;                 // accumulator columns of one tile
    constexpr uint32_t kCols = 2 * W;           // two accumulators
    extern __shared__ unsigned char pf_smem_raw[];
    const uint32_t raw = smem_u32(pf_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = pf_smem_raw + (base - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPfStages * kPfStage);
    uint64_t* empty = full + kPfStages;
    uint64_t* acc_full = empty + kPfStages;     // [2] MMA -> epilogue
    uint64_t* acc_empty = acc_full + 2;         // [2] epilogue (4 warps) -> MMA
    uint64_t* drain = acc_empty + 2;            // every MMA issued has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued = const_cast<int*>(abort_flag) + 1;
    int* consumed = issued + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int it0 = sk_begin(a, blockIdx.x), it1 = sk_begin(a, blockIdx.x + 1);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kPfStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        *issued = 0;
        *consumed = 0;
        fence_barrier_init();
    }
    if (warp == 2) tmem_alloc(tmem_slot, kCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();   // (programmatic launch) the activations come from the previous kernel
    pdl_launch_dependents();

    if (warp == 0 && lane == 0) {
        // ---- producer: one TMA ring through all segments -----------------------------
        prefetch_tmap(&maps.xh);
        if (a.use_lo) prefetch_tmap(&maps.xl);
        int i = 0;
        bool ok = true;
        for (int it = it0; it < it1 && ok;) {
            const PfSeg g = pf_seg(a, it, it1);
            it += g.nkb;
            const int tile = g.u / a.sk_mtiles, s0 = (g.u - tile * a.sk_mtiles) * kPfBM;
            int mi[2] = {0, 0}, row[2] = {0, 0};
            bool hv[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) hv[h] = h < NH && pf_half(a, NH, tile, h, mi[h], row[h]);
            const uint32_t bytes =
                (uint32_t)(kPfPlane * (a.use_lo ? 2 : 1) + (hv[0] ? kPfHalf : 0) + (hv[1] ? kPfHalf : 0));
            for (int k = 0; k < g.nkb; ++k, ++i) {
                const int s = i % kPfStages, r = i / kPfStages, kx = (g.kb0 + k) * kPfBK;
                if (r > 0 && !mbar_wait_bounded(&empty[s], (uint32_t)((r - 1) & 1))) {
                    pf_fail(a, abort_flag);
                    ok = false;
                    break;
                }
                if (*abort_flag) {
                    ok = false;
                    break;
                }
                const uint32_t st = base + (uint32_t)(s * kPfStage);
                mbar_expect_tx(&full[s], bytes);
                tma_load_2d(st, &maps.xh, kx, s0, &full[s]);
                if (a.use_lo) tma_load_2d(st + kPfPlane, &maps.xl, kx, s0, &full[s]);
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    if (hv[h]) tma_load_2d(st + 2 * kPfPlane + h * kPfHalf, &maps.w[mi[h]], kx, row[h], &full[s]);
            }
        }
        *issued = i;
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer: accumulator j & 1 for segment j -----------------------------
        constexpr uint32_t idesc = umma_idesc_f16(kPfBM, W);
        int i = 0, j = 0;
        bool ok = true;
        for (int it = it0; it < it1 && ok; ++j) {
            const PfSeg g = pf_seg(a, it, it1);
            it += g.nkb;
            const int buf = j & 1;
            if (j >= 2 && !mbar_wait_bounded(&acc_empty[buf], (uint32_t)(((j >> 1) - 1) & 1))) {
                pf_fail(a, abort_flag);
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(buf * W);
            for (int k = 0; k < g.nkb; ++k) {
                const int s = i % kPfStages, r = i / kPfStages;
                if (!mbar_wait_bounded(&full[s], (uint32_t)(r & 1))) {
                    pf_fail(a, abort_flag);
                    ok = false;
                    break;
                }
                ++i;
                tc_fence_after();
                const uint32_t st = base + (uint32_t)(s * kPfStage);
#pragma unroll
                for (int kk = 0; kk < kPfBK / 16; ++kk) {
                    const uint64_t bdesc = sw128_desc(st + 2 * kPfPlane + kk * 32);
                    tc_mma(d, sw128_desc(st + kk * 32), bdesc, idesc, (k | kk) != 0 ? 1u : 0u);
                    if (a.use_lo) tc_mma(d, sw128_desc(st + kPfPlane + kk * 32), bdesc, idesc, 1u);
                }
                tc_commit(&empty[s]);   // stage s is free once these MMAs have read it
            }
            tc_commit(&acc_full[buf]);  // (also after a failure: the epilogue sees the abort flag)
        }
        *consumed = i;
        tc_commit(drain);
        if (!mbar_wait_bounded(drain, 0u)) pf_fail(a, abort_flag);
    } else if (warp >= 4) {
        // ---- epilogue: warp q owns TMEM lanes (token rows) 32q .. 32q + 31 -----------
        const int q = warp & 3;
        const uint32_t ob = base + (uint32_t)(kPfStages * kPfStage + kPfBarBytes + q * 2 * kPfOutStage);
        PfEmit out{&maps, {ob, ob + (uint32_t)kPfOutStage}, 0, lane, a.tma_out != 0, true};
        int j = 0;
        for (int it = it0; it < it1; ++j) {
            const PfSeg g = pf_seg(a, it, it1);
            it += g.nkb;
            const int buf = j & 1;
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const int tile = g.u / a.sk_mtiles, s_base = (g.u - tile * a.sk_mtiles) * kPfBM + 32 * q;
            int mi[2] = {0, 0}, row[2] = {0, 0};
            bool hv[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) hv[h] = h < NH && pf_half(a, NH, tile, h, mi[h], row[h]);
            if (!g.piece) pf_epilogue_prefetch<NH>(a, s_base, lane);
            const bool got = __all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[buf], (uint32_t)((j >> 1) & 1)));
            tc_fence_after();
            if (!got) {
                if (lane == 0) pf_fail(a, abort_flag);
                break;
            }
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;   // the sums may be incomplete
            const uint32_t trow = tmem + (uint32_t)(buf * W) + ((uint32_t)(32 * q) << 16);
            const float e2 = pf_e2(a, s_base + lane);
            // this lane's row of accumulator columns [col, col + 32), times 2^row_exp
            auto tm = [&](int col, float (&v)[32]) {
                uint32_t r0[32];
                tmem_ld32(trow + col, r0);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < 32; ++t) v[t] = __uint_as_float(r0[t]) * e2;
            };
            if (g.piece) {
                // the warp's 32 rows (scaled): each 32-column chunk as 8
                // float4 slices of 32 lanes, so every store is 512 contiguous bytes
                float4* dst = reinterpret_cast<float4*>(a.part) + pf_piece_idx(blockIdx.x, q, 0, W, lane);
                float v[32];
                for (int c = 0; c < W / 32; ++c) {
                    tm(c * 32, v);
#pragma unroll
                    for (int t = 0; t < 8; ++t)
                        dst[(c * 8 + t) * 32] = make_float4(v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]);
                }
                // the warp's rows are stored: publish them (release orders the
                // whole warp's stores, which __syncwarp makes this lane's)
                __syncwarp();
                if (lane == 0) {
                    __threadfence();
                    st_release_gpu(a.sk_flags + (size_t)blockIdx.x * 4 + q, a.sk_epoch);
                }
            } else {
                bool fine = true;
                for (int h = 1; h <= g.helpers && fine; ++h) {
                    const unsigned* f = a.sk_flags + (size_t)(blockIdx.x + h) * 4 + q;
                    const long long t0 = clock64();
                    while (ld_acquire_u32_gpu(f) != a.sk_epoch) {
                        if (*abort_flag || clock64() - t0 > kSpinLimitCycles) {
                            fine = false;
                            break;
                        }
                    }
                }
                if (!__all_sync(0xffffffffu, fine)) {
                    if (lane == 0) pf_fail(a, abort_flag);
                    break;
                }
                out.srow = s_base + lane < a.S;
                // the later pieces of this unit (slots blockIdx.x + 1 .., this
                // lane's row, stored scaled), added in k order
                const int helpers = g.helpers;
                pf_tile_epilogue<NH>(a, s_base, lane, mi, row, hv, [&](int col, float (&v)[32]) {
                    tm(col, v);
                    for (int h = 0; h < helpers; ++h) {
                        const float4* p4 = reinterpret_cast<const float4*>(a.part) +
                                           pf_piece_idx(blockIdx.x + 1 + h, q, col / 32, W, lane);
                        float4 x[8];
#pragma unroll
                        for (int t = 0; t < 8; ++t) x[t] = __ldcg(p4 + t * 32);
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            v[4 * t] = __fadd_rn(v[4 * t], x[t].x);
                            v[4 * t + 1] = __fadd_rn(v[4 * t + 1], x[t].y);
                            v[4 * t + 2] = __fadd_rn(v[4 * t + 2], x[t].z);
                            v[4 * t + 3] = __fadd_rn(v[4 * t + 3], x[t].w);
                        }
                    }
                }, out);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        out.finish();
    }
    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        // leave no TMA write in flight into this CTA's shared memory
        for (int kb = *consumed; kb < *issued; ++kb)
            mbar_wait_bounded(&full[kb % kPfStages], (uint32_t)((kb / kPfStages) & 1));
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
}

// ---------------------------------------------------------------------------
// Few activation rows (S <= 16: batched decode, short chunks): the operands
// swap roles so the MMA is M = 128 weight rows x N = 16 rows of x.  With the
// tokens as M (pf_gemm_kernel) a 128-row MMA would compute 112+ empty token
// rows per weight tile; here the tensor work per weight byte is 8x smaller and
// the shared memory holds 6 weight stages in flight instead of 3.  TMEM: 32
// columns, half h (128 weight rows) in columns [16h, 16h + 16), column = row
// of x; warp w of the epilogue reads TMEM lanes 32*(w%4).. = its weight rows.
// ---------------------------------------------------------------------------
constexpr int kPsN = 16;                        // rows of x per MMA (N)
constexpr int kPsStages = 6;
constexpr int kPsPlane = kPsN * kPfBK * 2;      // 2 KB activation plane per stage
__host__ __device__ constexpr int ps_stage_bytes(int nh) { return 2 * kPsPlane + nh * kPfHalf; }
__host__ __device__ constexpr int ps_smem_bytes(int nh) { return kPsStages * ps_stage_bytes(nh) + 1024 + 256; }

template <int NH>
__global__ void __launch_bounds__(kPfThreads, 1)
pf_gemm_small_kernel(const __grid_constant__ PfMaps maps, const __grid_constant__ PfArgs a) {
    constexpr int kStage = ps_stage_bytes(NH);
    constexpr uint32_t kTmemCols = 32;
    extern __shared__ unsigned char ps_smem_raw[];
    const uint32_t raw = smem_u32(ps_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = ps_smem_raw + (base - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPsStages * kStage);
    uint64_t* empty = full + kPsStages;
    uint64_t* done = empty + kPsStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued = const_cast<int*>(abort_flag) + 1;
    int* consumed = issued + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    const int kb0 = (int)((long long)a.nk * blockIdx.z / gridDim.z);
    const int nkb = (int)((long long)a.nk * (blockIdx.z + 1) / gridDim.z) - kb0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kPsStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        *issued = 0;
        *consumed = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    if (!(warp == 0 && lane == 0)) pdl_wait();   // the producer waits after its first weight requests

    int mi[2], row[2];
    bool hv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) hv[h] = h < NH && pf_half(a, NH, tile, h, mi[h], row[h]);

    if (warp == 0 && lane == 0) {
        // ---- producer: TMA ring (x planes: 16 rows; weight halves: 128 rows) -----
        prefetch_tmap(&maps.xh);
        if (a.use_lo) prefetch_tmap(&maps.xl);
        const uint32_t bytes =
            (uint32_t)(kPsPlane * (a.use_lo ? 2 : 1) + (hv[0] ? kPfHalf : 0) + (hv[1] ? kPfHalf : 0));
        // Programmatic launch: weights that no earlier kernel of the stream
        // writes are requested for the first stages before the wait for the
        // previous kernel (whose output is x); then x for those stages.
        const int pre = a.w_static ? (nkb < kPsStages ? nkb : kPsStages) : 0;
        for (int j = 0; j < pre; ++j) {
            const uint32_t st = base + (uint32_t)(j * kStage);
            mbar_expect_tx(&full[j], bytes);
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (hv[h])
                    tma_load_2d(st + 2 * kPsPlane + h * kPfHalf, &maps.w[mi[h]], (kb0 + j) * kPfBK, row[h], &full[j]);
        }
        pdl_wait();
        for (int j = 0; j < pre; ++j) {
            const uint32_t st = base + (uint32_t)(j * kStage);
            tma_load_2d(st, &maps.xh, (kb0 + j) * kPfBK, 0, &full[j]);
            if (a.use_lo) tma_load_2d(st + kPsPlane, &maps.xl, (kb0 + j) * kPfBK, 0, &full[j]);
        }
        int i = pre;
        for (; i < nkb; ++i) {
            const int s = i % kPsStages, r = i / kPsStages, kx = (kb0 + i) * kPfBK;
            if (r > 0 && !mbar_wait_bounded(&empty[s], (uint32_t)((r - 1) & 1))) {
                pf_fail(a, abort_flag);
                break;
            }
            if (*abort_flag) break;
            const uint32_t st = base + (uint32_t)(s * kStage);
            mbar_expect_tx(&full[s], bytes);
            tma_load_2d(st, &maps.xh, kx, 0, &full[s]);
            if (a.use_lo) tma_load_2d(st + kPsPlane, &maps.xl, kx, 0, &full[s]);
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (hv[h]) tma_load_2d(st + 2 * kPsPlane + h * kPfHalf, &maps.w[mi[h]], kx, row[h], &full[s]);
        }
        *issued = i;
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer: D[weight row][x row] += W . X^T per half ----------------------
        constexpr uint32_t idesc = umma_idesc_f16(128, kPsN);
        int kb = 0;
        for (; kb < nkb; ++kb) {
            const int s = kb % kPsStages, r = kb / kPsStages;
            if (!mbar_wait_bounded(&full[s], (uint32_t)(r & 1))) {
                pf_fail(a, abort_flag);
                break;
            }
            tc_fence_after();
            const uint32_t st = base + (uint32_t)(s * kStage);
#pragma unroll
            for (int kk = 0; kk < kPfBK / 16; ++kk) {
                const uint64_t xhd = sw128_desc(st + kk * 32);
                const uint64_t xld = sw128_desc(st + kPsPlane + kk * 32);
#pragma unroll
                for (int h = 0; h < NH; ++h) {
                    if (!hv[h]) continue;
                    const uint64_t wd = sw128_desc(st + 2 * kPsPlane + h * kPfHalf + kk * 32);
                    tc_mma(tmem + (uint32_t)(h * kPsN), wd, xhd, idesc, (kb | kk) != 0 ? 1u : 0u);
                    if (a.use_lo) tc_mma(tmem + (uint32_t)(h * kPsN), wd, xld, idesc, 1u);
                }
            }
            tc_commit(&empty[s]);
        }
        *consumed = kb;
        tc_commit(done);
    } else if (warp >= 4) {
        // ---- epilogue: thread = weight row r of each half, its 16 columns = rows of x --
        const int q = warp & 3;
        const int r = 32 * q + lane;
        const bool ok = mbar_wait_bounded(done, 0u);
        tc_fence_after();
        if (!ok) pf_fail(a, abort_flag);
        uint32_t acc[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16), acc);
        tmem_wait_ld();
        const bool run = ok && !*abort_flag;
        const int S = a.S;
        float e2[kPsN];
#pragma unroll
        for (int t = 0; t < kPsN; ++t) e2[t] = (t < S && a.row_exp) ? ldexpf(1.0f, __ldg(a.row_exp + t)) : 1.0f;
        if (gridDim.z > 1) {
            if (run) {
#pragma unroll
                for (int h = 0; h < NH; ++h) {
                    if (!hv[h]) continue;
                    float* dst = a.part + (size_t)blockIdx.z * S * a.width + (size_t)tile * 128 * NH + h * 128 + r;
#pragma unroll
                    for (int t = 0; t < kPsN; ++t)
                        if (t < S) dst[(size_t)t * a.width] = __uint_as_float(acc[h * kPsN + t]);
                }
            }
        } else if (a.mode == PF_GATEUP) {
            // relu2_d then mul_d (ops_cuda.cu:123-130, 116-121)
            const int n = row[0] + r;
            if (run && hv[0] && hv[1] && n < a.rows[0]) {
                const float sg = pf_row_scale(a, 0, n), su = pf_row_scale(a, 1, n);
#pragma unroll
                for (int t = 0; t < kPsN; ++t) {
                    if (t >= S) continue;
                    const float g = __fmul_rn(__uint_as_float(acc[t]) * e2[t], sg);
                    const float u = __fmul_rn(__uint_as_float(acc[kPsN + t]) * e2[t], su);
                    const float gr = fmaxf(g, 0.0f);
                    a.y[(size_t)t * a.ldy + n] = __fmul_rn(__fmul_rn(gr, gr), u);
                }
            }
        } else if (a.mode == PF_QKV) {
            // RoPE pairs rows (d, d + 64) of a head, held by warps q and q + 2:
            // exchange through shared memory (the pipeline's stages are idle now)
            float* ex = reinterpret_cast<float*>(smem);   // [NH][128][kPsN + 1]
#pragma unroll
            for (int h = 0; h < NH; ++h)
#pragma unroll
                for (int t = 0; t < kPsN; ++t) ex[(h * 128 + r) * (kPsN + 1) + t] = __uint_as_float(acc[h * kPsN + t]);
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const int half = a.hd >> 1;
            if (run && r < half) {
                const int d = r;
#pragma unroll
                for (int h = 0; h < NH; ++h) {
                    if (!hv[h]) continue;
                    const int head = row[h] / a.hd;
                    const float s0 = pf_row_scale(a, mi[h], row[h] + d);
                    const float s1 = pf_row_scale(a, mi[h], row[h] + d + half);
                    for (int t = 0; t < S; ++t) {
                        const int pos = pf_pos(a, t);
                        float y0 = __fmul_rn(ex[(h * 128 + d) * (kPsN + 1) + t] * e2[t], s0);
                        float y1 = __fmul_rn(ex[(h * 128 + d + half) * (kPsN + 1) + t] * e2[t], s1);
                        if (mi[h] < 2) {
                            // NeoX pair (d, d + hd/2), tensor.cpp:918-925
                            const float cs = __ldg(a.rope_cos + (size_t)pos * half + d);
                            const float sn = __ldg(a.rope_sin + (size_t)pos * half + d);
                            const float t0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                            const float t1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
                            y0 = t0;
                            y1 = t1;
                        }
                        float* dst = mi[h] == 0 ? a.q_out + (size_t)t * a.nh * a.hd + head * a.hd
                                                : (mi[h] == 1 ? a.kcache : a.vcache) + pf_slot(a, t) +
                                                      (size_t)pos * a.nkv * a.hd + head * a.hd;
                        dst[d] = y0;
                        dst[d + half] = y1;
                    }
                }
            }
        } else {
            const bool add = a.mode == PF_RESID;
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                const int n = row[h] + r;
                if (!run || !hv[h] || n >= a.rows[0]) continue;
                const float sc = pf_row_scale(a, 0, n);
#pragma unroll
                for (int t = 0; t < kPsN; ++t) {
                    if (t >= S) continue;
                    const float v = __fmul_rn(__uint_as_float(acc[h * kPsN + t]) * e2[t], sc);
                    float* y = a.y + (size_t)t * a.ldy + n;
                    *y = add ? __fadd_rn(*y, v) : v;
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        for (int kb = *consumed; kb < *issued; ++kb)
            mbar_wait_bounded(&full[kb % kPsStages], (uint32_t)((kb / kPsStages) & 1));
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// Split-K completion: one thread per (row, output element or RoPE/gate-up
// pair): the ksplit partial sums added in split order, then the epilogue of
// pf_gemm_kernel (same arithmetic after the sum).
template <int NH>
__global__ void pf_splitk_epilogue(const __grid_constant__ PfArgs a) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (idx >= (size_t)a.S * a.width) return;
    const int s = (int)(idx / a.width), v = (int)(idx % a.width);
    const int tile = v / (128 * NH), h = (v / 128) % NH, c = v % 128;
    int mi, row;
    if (!pf_half(a, NH, tile, h, mi, row)) return;
    const size_t plane = (size_t)a.S * a.width;
    auto sum = [&](int col) {
        const float* p = a.part + (size_t)s * a.width + col;
        float t = 0.f;
        for (int z = 0; z < a.ksplit; ++z) t += p[z * plane];
        return t;
    };
    const float e2 = a.row_exp ? ldexpf(1.0f, a.row_exp[s]) : 1.0f;
    if (a.mode == PF_GATEUP) {
        // the gate half (h 0) finishes the pair with its up half (h 1)
        const int n = row + c;
        if (h != 0 || n >= a.rows[0]) return;
        const float g = __fmul_rn(sum(v) * e2, pf_row_scale(a, 0, n));
        const float u = __fmul_rn(sum(v + 128) * e2, pf_row_scale(a, 1, n));
        const float gr = fmaxf(g, 0.0f);
        a.y[(size_t)s * a.ldy + n] = __fmul_rn(__fmul_rn(gr, gr), u);
    } else if (a.mode == PF_QKV) {
        const int half = a.hd >> 1;
        if (c >= half) return;
        const int head = row / a.hd, pos = pf_pos(a, s);
        float y0 = __fmul_rn(sum(v) * e2, pf_row_scale(a, mi, row + c));
        float y1 = __fmul_rn(sum(v + half) * e2, pf_row_scale(a, mi, row + c + half));
        if (mi < 2) {
            // NeoX pair (d, d + hd/2), tensor.cpp:918-925
            const float cs = __ldg(a.rope_cos + (size_t)pos * half + c);
            const float sn = __ldg(a.rope_sin + (size_t)pos * half + c);
            const float t0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
            const float t1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
            y0 = t0;
            y1 = t1;
        }
        float* dst = mi == 0 ? a.q_out + (size_t)s * a.nh * a.hd + head * a.hd
                             : (mi == 1 ? a.kcache : a.vcache) + pf_slot(a, s) + (size_t)pos * a.nkv * a.hd +
                                   head * a.hd;
        dst[c] = y0;
        dst[c + half] = y1;
    } else {
        const int n = row + c;
        if (n >= a.rows[0]) return;
        const float val = __fmul_rn(sum(v) * e2, pf_row_scale(a, 0, n));
        float* y = a.y + (size_t)s * a.ldy + n;
        *y = a.mode == PF_RESID ? __fadd_rn(*y, val) : val;
    }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launch
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn(tvb_status* st) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    *st = fn ? TVB_OK : set_error(TVB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

tvb_status encode_f16_tiled(CUtensorMap* m, const void* p, int rank, const uint64_t* dims, const uint64_t* strides,
                            const uint32_t* box, CUtensorMapSwizzle swizzle) {
    tvb_status st;
    auto fn = encode_fn(&st);
    if (!fn) return st;
    TVB_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15) == 0, "tensor map: base not 16-byte aligned");
    cuuint64_t d[5], sb[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1u;
        if (i + 1 < rank) sb[i] = strides[i];
    }
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank, const_cast<void*>(p), d, sb, b, e,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(TVB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TVB_OK;
}

// F16 matrix [rows][K] (row pitch K), boxes of 128 rows x 64 k, 128B swizzle.
static tvb_status encode_f16(CUtensorMap* m, const void* p, int rows, int K, int box_rows = 128) {
    tvb_status st;
    auto fn = encode_fn(&st);
    if (!fn) return st;
    TVB_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15) == 0, "prefill gemm: operand not 16-byte aligned");
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kPfBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(TVB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TVB_OK;
}

// F32 output matrix [rows][cols] (row pitch stride_bytes) for the epilogue's
// TMA stores: 32 x 32 boxes, 128-byte swizzle (matching PfEmit's shared boxes).
static tvb_status encode_f32_out(CUtensorMap* m, const float* p, int cols, int rows, size_t stride_bytes) {
    tvb_status st;
    auto fn = encode_fn(&st);
    if (!fn) return st;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride_bytes};
    const cuuint32_t box[2] = {32u, 32u};
    const cuuint32_t estr[2] = {1u, 1u};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(TVB_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
    return TVB_OK;
}

// The epilogue writes through TMA when every output matrix has a 16-byte
// aligned base and row pitch (and the K/V rows of a QKV tile are consecutive
// positions); otherwise through per-thread stores.
static bool pf_out_aligned(const void* p, size_t pitch_bytes) {
    return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && pitch_bytes % 16 == 0;
}

static tvb_status pf_prepare() {
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    std::call_once(once, [] {
        err = cudaFuncSetAttribute(pf_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf_smem_bytes(2));
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(pf_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       pf_smem_bytes(1));
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(pf_gemm_sk_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       pf_smem_bytes(2));
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(pf_gemm_sk_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       pf_smem_bytes(1));
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(pf_gemm_small_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       ps_smem_bytes(2));
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(pf_gemm_small_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       ps_smem_bytes(1));
    });
    if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(pf_gemm_kernel)");
    return TVB_OK;
}

tvb_status pf_gemm(const PfGemm& g, cudaStream_t stream) {
    TVB_REQUIRE(g.S > 0 && g.K > 0 && g.xh, "prefill gemm: empty problem");
    TVB_REQUIRE(g.K % kPfBK == 0, "prefill gemm: K=%d must be a multiple of %d", g.K, kPfBK);
    TVB_TRY(pf_prepare());
    PfMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    PfArgs a;
    std::memset(&a, 0, sizeof(a));
    a.mode = g.mode;
    a.S = g.S;
    a.K = g.K;
    a.nk = g.K / kPfBK;
    a.use_lo = g.xl != nullptr;
    a.row_exp = g.row_exp;
    a.y = g.y;
    a.ldy = g.ldy;
    a.nh = g.nh;
    a.nkv = g.nkv;
    a.hd = g.hd;
    a.pos0 = g.pos0;
    a.q_out = g.q_out;
    a.kcache = g.kcache;
    a.vcache = g.vcache;
    a.rope_cos = g.rope_cos;
    a.rope_sin = g.rope_sin;
    a.row_pos = g.row_pos;
    a.kv_slot_stride = g.kv_slot_stride;
    a.status = g.status;
    const bool small = g.S <= kPsN;   // few rows of x: the swapped-operand kernel
    TVB_TRY(encode_f16(&maps.xh, g.xh, g.S, g.K, small ? kPsN : 128));
    if (g.xl) TVB_TRY(encode_f16(&maps.xl, g.xl, g.S, g.K, small ? kPsN : 128));
    const int nm = g.mode == PF_QKV ? 3 : g.mode == PF_GATEUP ? 2 : 1;
    a.w_static = 1;
    for (int i = 0; i < nm; ++i) {
        if (g.m[i].widened) a.w_static = 0;
        TVB_REQUIRE(g.m[i].w && g.m[i].rows > 0, "prefill gemm: matrix %d missing", i);
        TVB_TRY(encode_f16(&maps.w[i], g.m[i].w, g.m[i].rows, g.K));
        a.rows[i] = g.m[i].rows;
        a.row_scales[i] = g.m[i].row_scales;
        a.scale[i] = g.m[i].scale;
    }
    // 128-row halves of weight rows: q/k/v heads (one half each) or plain rows
    int halves = 0;
    if (g.mode == PF_QKV) {
        TVB_REQUIRE(g.hd == 128 && g.m[0].rows == g.nh * 128 && g.m[1].rows == g.nkv * 128 &&
                        g.m[2].rows == g.nkv * 128 && g.q_out && g.kcache && g.vcache && g.rope_cos && g.rope_sin,
                    "prefill gemm: inconsistent q/k/v geometry");
        halves = g.nh + 2 * g.nkv;
    } else if (g.mode == PF_GATEUP) {
        TVB_REQUIRE(g.m[0].rows == g.m[1].rows && g.m[0].rows % 32 == 0 && g.y && g.ldy >= g.m[0].rows,
                    "prefill gemm: gate/up shapes");
    } else {
        TVB_REQUIRE(g.y && g.ldy >= g.m[0].rows, "prefill gemm: output");
        halves = (g.m[0].rows + 127) / 128;
    }
    const int mtiles = (g.S + kPfBM - 1) / kPfBM;
    if (!small) {
        if (g.mode == PF_QKV) {
            const size_t qp = (size_t)g.nh * g.hd * 4, kp = (size_t)g.nkv * g.hd * 4;
            a.tma_out = !g.row_pos && pf_out_aligned(g.q_out, qp) && pf_out_aligned(g.kcache, kp) &&
                        pf_out_aligned(g.vcache, kp);
            if (a.tma_out) {
                TVB_TRY(encode_f32_out(&maps.out[0], g.q_out, g.nh * g.hd, g.S, qp));
                TVB_TRY(encode_f32_out(&maps.out[1], g.kcache, g.nkv * g.hd, g.pos0 + g.S, kp));
                TVB_TRY(encode_f32_out(&maps.out[2], g.vcache, g.nkv * g.hd, g.pos0 + g.S, kp));
            }
        } else {
            a.tma_out = pf_out_aligned(g.y, (size_t)g.ldy * 4);
            if (a.tma_out) TVB_TRY(encode_f32_out(&maps.out[0], g.y, g.m[0].rows, g.S, (size_t)g.ldy * 4));
        }
    }
    if (!small && g.part && g.flags) {
        // Long reductions whose tiles leave SMs idle but are cut into at most
        // four pieces (the down projection of a 512- or 1024-token chunk): the
        // persistent stream-K kernel, 256-row weight tiles (128 when the
        // matrices have a single 128-row half).  Measured at 1024 tokens of the
        // 2B shape, down 78.6 -> 69.6 us; q/k/v (40 k-blocks, 120 tiles) was
        // 45.5 us data-parallel against 54.9 us, o_proj and gate/up even.
        const int nh_sk = (g.mode == PF_GATEUP || halves > 1) ? 2 : 1;
        const int tiles_sk = g.mode == PF_GATEUP ? (g.m[0].rows + 127) / 128 : (halves + nh_sk - 1) / nh_sk;
        const long long units = (long long)tiles_sk * mtiles;
        const long long total = units * a.nk;
        const int G = (int)std::min<long long>(num_sms(), total);
        if (a.nk >= 64 && units < num_sms() && 4 * units >= G && total < (1LL << 31) &&
            (size_t)G * kPfBM * 128 * nh_sk <= g.part_floats) {
            static unsigned epoch = 0;   // flags of an earlier launch never match this one's
            if (++epoch == 0) epoch = 1;
            a.sk_total = (int)total;
            a.sk_mtiles = mtiles;
            a.sk_epoch = epoch;
            a.sk_flags = g.flags;
            a.part = g.part;
            const dim3 grid((unsigned)G), block(kPfThreads);
            const cudaError_t e = nh_sk == 2
                ? launch_maybe_pdl(pf_gemm_sk_kernel<2>, grid, block, pf_smem_bytes(2), stream, g.pdl, maps, a)
                : launch_maybe_pdl(pf_gemm_sk_kernel<1>, grid, block, pf_smem_bytes(1), stream, g.pdl, maps, a);
            if (e != cudaSuccess) return cuda_error(e, "launch pf_gemm_sk_kernel");
            return check_launch("pf_gemm_sk_kernel");
        }
    }
    // 256-row tiles, or 128-row tiles when those keep more of the SMs busy over
    // the grid's waves (gate/up tiles always pair a gate half with an up half)
    int nh = 2, tiles;
    if (g.mode == PF_GATEUP) {
        tiles = (g.m[0].rows + 127) / 128;
    } else {
        tiles = (halves + 1) / 2;
        const int sms = num_sms();
        auto busy = [&](int ctas) { return (double)ctas / (double)(((ctas + sms - 1) / sms) * sms); };
        if (busy(halves * mtiles) > busy(tiles * mtiles) + 1e-9) {
            nh = 1;
            tiles = halves;
        }
    }
    // split-K when the tiles leave most SMs idle (few activation rows): each
    // split keeps at least 8 k-blocks for its TMA/MMA pipeline
    int ksplit = 1;
    if (g.part) {
        const int sms = num_sms();
        ksplit = std::max(1, std::min(sms / (tiles * mtiles), a.nk / 8));
        a.width = tiles * 128 * nh;
        while (ksplit > 1 && (size_t)ksplit * g.S * a.width > g.part_floats) --ksplit;
        a.part = g.part;
        a.ksplit = ksplit;
    }
    const dim3 grid((unsigned)tiles, (unsigned)mtiles, (unsigned)ksplit);
    const dim3 block(kPfThreads);
    cudaError_t le;
    if (small && nh == 2) le = launch_maybe_pdl(pf_gemm_small_kernel<2>, grid, block, ps_smem_bytes(2), stream, g.pdl, maps, a);
    else if (small) le = launch_maybe_pdl(pf_gemm_small_kernel<1>, grid, block, ps_smem_bytes(1), stream, g.pdl, maps, a);
    else if (nh == 2) le = launch_maybe_pdl(pf_gemm_kernel<2>, grid, block, pf_smem_bytes(2), stream, g.pdl, maps, a);
    else le = launch_maybe_pdl(pf_gemm_kernel<1>, grid, block, pf_smem_bytes(1), stream, g.pdl, maps, a);
    if (le != cudaSuccess) return cuda_error(le, "launch pf_gemm_kernel");
    TVB_TRY(check_launch("pf_gemm_kernel"));
    if (ksplit == 1) return TVB_OK;
    const size_t n = (size_t)g.S * a.width;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (nh == 2) TVB_CUDA(launch_maybe_pdl(pf_splitk_epilogue<2>, dim3(blocks), dim3(256), 0, stream, g.pdl, a));
    else TVB_CUDA(launch_maybe_pdl(pf_splitk_epilogue<1>, dim3(blocks), dim3(256), 0, stream, g.pdl, a));
    return check_launch("pf_splitk_epilogue");
}

// ---------------------------------------------------------------------------
// RMSNorm + hi/lo split, embedding gather, INT8 widening
// ---------------------------------------------------------------------------
// one CTA per row: 256 threads, or 1024 when the rows alone leave most SMs idle

// The row is read once into registers (at most MAXV float4 per thread), then
// reduced twice (sum of squares, largest magnitude) and written; the sums run
// in the same order as a strided pass over global memory would.
template <int NT, int MAXV>
__global__ void __launch_bounds__(NT)
pf_norm_split_kernel(const float* __restrict__ x, const float* __restrict__ w, int K, float eps,
                     __half* __restrict__ xh, __half* __restrict__ xl, int* __restrict__ row_exp,
                     float* __restrict__ ss_out) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const int row = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)row * K);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const int K4 = K >> 2;
    __shared__ float red[NT / 32];
    __shared__ float s_inv, s_max;
    float4 v[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int k = tid + i * NT;
        v[i] = k < K4 ? x4[k] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    float inv = 1.0f;
    if (w) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
            for (int i = 0; i < NT / 32; ++i) t += red[i];
            // tensor.cpp:672-673: rms = sqrt(ss/n + eps); inv_rms = 1/rms.  A
            // sub-norm whose row spans the tensor-parallel ranks is deferred:
            // the row's sum of squares goes out and the consumer scales by the
            // factor of the ranks' summed squares.
            if (ss_out) {
                ss_out[row] = t;
                s_inv = 1.0f;
            } else {
                s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), eps)));
            }
        }
        __syncthreads();
        inv = s_inv;
    }
    // the normalised row x * (inv_rms * w) (the vectorised path of tensor_rms_norm)
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int k = tid + i * NT;
        if (k < K4 && w) {
            const float4 g = w4[k];
            v[i] = make_float4(v[i].x * (inv * g.x), v[i].y * (inv * g.y), v[i].z * (inv * g.z),
                               v[i].w * (inv * g.w));
        }
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
    mx = warp_max(mx);
    __syncthreads();
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < NT / 32; ++i) t = fmaxf(t, red[i]);
        s_max = t;
    }
    __syncthreads();
    // power-of-two row scale: largest magnitude into [2^14, 2^15) (rows below
    // 2^-86 stay scaled by 2^100, which keeps 2^-e finite)
    const int e = (s_max > 0.f && isfinite(s_max)) ? max(ilogbf(s_max) - 14, -100) : 0;
    if (tid == 0) row_exp[row] = e;
    const float sc = ldexpf(1.0f, -e);
    uint2* h2 = reinterpret_cast<uint2*>(xh + (size_t)row * K);
    uint2* l2 = reinterpret_cast<uint2*>(xl + (size_t)row * K);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int k = tid + i * NT;
        if (k >= K4) continue;
        const float f[4] = {v[i].x * sc, v[i].y * sc, v[i].z * sc, v[i].w * sc};
        __half hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            hi[j] = __float2half_rn(f[j]);
            lo[j] = __float2half_rn(f[j] - __half2float(hi[j]));
        }
        const __half2 h01 = __halves2half2(hi[0], hi[1]), h23 = __halves2half2(hi[2], hi[3]);
        const __half2 l01 = __halves2half2(lo[0], lo[1]), l23 = __halves2half2(lo[2], lo[3]);
        h2[k] = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
        l2[k] = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
    }
}

__global__ void pf_embed_kernel(const uint16_t* __restrict__ embd, const int* __restrict__ tokens, int H,
                                float* __restrict__ x) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const int s = blockIdx.x;
    const uint16_t* e = embd + (size_t)__ldg(tokens + s) * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x)
        x[(size_t)s * H + k] = __half2float(__ushort_as_half(__ldg(e + k)));
}

__global__ void pf_i8_kernel(const int8_t* __restrict__ q, size_t n, __half* __restrict__ out) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const size_t n4 = n >> 2;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const char4 c = reinterpret_cast<const char4*>(q)[i];
        reinterpret_cast<__half2*>(out)[2 * i] = __halves2half2(__int2half_rn(c.x), __int2half_rn(c.y));
        reinterpret_cast<__half2*>(out)[2 * i + 1] = __halves2half2(__int2half_rn(c.z), __int2half_rn(c.w));
    }
}

tvb_status pf_norm_split(const float* x, const float* w, int S, int K, float eps, uint16_t* xh, uint16_t* xl,
                         int* row_exp, cudaStream_t st, float* ss_out, bool pdl) {
    TVB_REQUIRE(x && xh && xl && row_exp && S > 0 && K > 0 && K % 4 == 0, "norm_split: bad arguments");
    __half* h = reinterpret_cast<__half*>(xh);
    __half* l = reinterpret_cast<__half*>(xl);
    // one CTA per row; 1024 threads when the rows alone leave most SMs idle.
    // The row lives in registers: up to 16 float4 a thread with 256 threads
    // (K <= 16384), 8 with 1024 (K <= 32768)
    TVB_REQUIRE(K <= (S < num_sms() ? 8 * 4 * 1024 : 16 * 4 * 256), "norm_split: K=%d too long for a register row",
                K);
    if (S < num_sms())
        TVB_CUDA(launch_maybe_pdl(pf_norm_split_kernel<1024, 8>, dim3(S), dim3(1024), 0, st, pdl, x, w, K, eps,
                                  h, l, row_exp, ss_out));
    else if (K <= 8 * 4 * 256)
        TVB_CUDA(launch_maybe_pdl(pf_norm_split_kernel<256, 8>, dim3(S), dim3(256), 0, st, pdl, x, w, K, eps, h,
                                  l, row_exp, ss_out));
    else
        TVB_CUDA(launch_maybe_pdl(pf_norm_split_kernel<256, 16>, dim3(S), dim3(256), 0, st, pdl, x, w, K, eps, h,
                                  l, row_exp, ss_out));
    return check_launch("pf_norm_split_kernel");
}

tvb_status pf_embed(const uint16_t* embd, const int* tokens, int S, int H, float* x, cudaStream_t st, bool pdl) {
    TVB_REQUIRE(embd && tokens && x && S > 0 && H > 0, "embed: bad arguments");
    TVB_CUDA(launch_maybe_pdl(pf_embed_kernel, dim3(S), dim3(256), 0, st, pdl, embd, tokens, H, x));
    return check_launch("pf_embed_kernel");
}

tvb_status pf_i8_to_f16(const int8_t* q, size_t n, uint16_t* out, cudaStream_t st, bool pdl) {
    TVB_REQUIRE(q && out && n % 4 == 0, "i8_to_f16: bad arguments");
    const int blocks = (int)std::min<size_t>((n / 4 + 255) / 256, (size_t)num_sms() * 8);
    TVB_CUDA(launch_maybe_pdl(pf_i8_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, st, pdl, q, n,
                              reinterpret_cast<__half*>(out)));
    return check_launch("pf_i8_kernel");
}

// ---------------------------------------------------------------------------
// Causal GQA attention (FP32 on the CUDA cores)
// ---------------------------------------------------------------------------
// A CTA takes one KV head and a block of query positions; its 64 rows are the
// (position, query head) pairs that share that KV head.  Keys stream through
// shared memory 64 at a time; each thread owns 4 rows x 4 keys of the score
// tile (keys j, j+16, j+32, j+48: conflict-free rows of the padded K tile) and
// 4 rows x 8 dims of the output, with online softmax (running max and sum per
// row, kept by the 16 threads that share the rows).
constexpr int kPaRows = 64, kPaKeys = 64, kPaThreads = 256;
constexpr int kPaQs = 132;   // padded row stride (floats) of the Q and K tiles
constexpr int kPaPs = 68;    // padded row stride of the probability tile
constexpr int kPaSmem = (kPaRows * kPaQs + kPaKeys * kPaQs + kPaKeys * 128) * 4;

__global__ void __launch_bounds__(kPaThreads, 2)
pf_attn_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc, int S,
               int pos0, int nh, int nkv, float scale, float* __restrict__ out) {
    extern __shared__ __align__(16) float pa_smem[];
    float* Qs = pa_smem;                      // [64 rows][132]
    float* Ks = Qs + kPaRows * kPaQs;         // [64 keys][132], reused for P [64 rows][68]
    float* Vs = Ks + kPaKeys * kPaQs;         // [64 keys][128]
    float* Ps = Ks;
    constexpr int hd = 128;
    const int group = nh / nkv, bq = kPaRows / group;
    const int kvh = blockIdx.x;
    const int qb = gridDim.y - 1 - blockIdx.y;   // longest blocks first
    const int qlo = qb * bq;                     // first query row (0-based within the prompt)
    const int tid = threadIdx.x, i = tid >> 4, j = tid & 15;
    const int Hq = nh * hd, Hk = nkv * hd;

    // Q tile: row r = (position qlo + r / group, head kvh * group + r % group)
    for (int idx = tid; idx < kPaRows * (hd / 4); idx += kPaThreads) {
        const int r = idx / (hd / 4), d4 = idx - r * (hd / 4);
        const int sq = qlo + r / group;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (sq < S) v = *reinterpret_cast<const float4*>(q + (size_t)sq * Hq + (kvh * group + r % group) * hd + d4 * 4);
        *reinterpret_cast<float4*>(Qs + r * kPaQs + d4 * 4) = v;
    }
    float m[4], l[4], o[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        m[a] = -INFINITY;
        l[a] = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) o[a][d] = 0.f;
    }
    int rpos[4];   // absolute position of each of this thread's rows (-1: none)
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int sq = qlo + (4 * i + a) / group;
        rpos[a] = sq < S ? pos0 + sq : -1;
    }
    const int last = pos0 + min(S, qlo + bq) - 1;   // largest position of this block
    for (int t0 = 0; t0 <= last; t0 += kPaKeys) {
        __syncthreads();   // previous tile's P and V reads are done
        for (int idx = tid; idx < kPaKeys * (hd / 4); idx += kPaThreads) {
            const int t = idx / (hd / 4), d4 = idx - t * (hd / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (t0 + t <= last) {
                kv = *reinterpret_cast<const float4*>(kc + (size_t)(t0 + t) * Hk + kvh * hd + d4 * 4);
                vv = *reinterpret_cast<const float4*>(vc + (size_t)(t0 + t) * Hk + kvh * hd + d4 * 4);
            }
            *reinterpret_cast<float4*>(Ks + t * kPaQs + d4 * 4) = kv;
            *reinterpret_cast<float4*>(Vs + t * 128 + d4 * 4) = vv;
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) sc[a][b] = 0.f;
#pragma unroll 4
        for (int d = 0; d < hd; d += 4) {
            float4 qa[4], kb4[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) qa[a] = *reinterpret_cast<const float4*>(Qs + (4 * i + a) * kPaQs + d);
#pragma unroll
            for (int b = 0; b < 4; ++b) kb4[b] = *reinterpret_cast<const float4*>(Ks + (j + 16 * b) * kPaQs + d);
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    sc[a][b] = fmaf(qa[a].x, kb4[b].x, sc[a][b]);
                    sc[a][b] = fmaf(qa[a].y, kb4[b].y, sc[a][b]);
                    sc[a][b] = fmaf(qa[a].z, kb4[b].z, sc[a][b]);
                    sc[a][b] = fmaf(qa[a].w, kb4[b].w, sc[a][b]);
                }
        }
        // online softmax over this tile (16 threads share each row)
        float alpha[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float tmax = -INFINITY;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int t = t0 + j + 16 * b;
                sc[a][b] = (t <= rpos[a]) ? sc[a][b] * scale : -INFINITY;
                tmax = fmaxf(tmax, sc[a][b]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mn = fmaxf(m[a], tmax);
            alpha[a] = (mn == -INFINITY) ? 1.f : expf(m[a] - mn);
            float psum = 0.f;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const float p = (mn == -INFINITY) ? 0.f : expf(sc[a][b] - mn);
                sc[a][b] = p;
                psum += p;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l[a] = l[a] * alpha[a] + psum;
            m[a] = mn;
        }
        __syncthreads();   // everyone is done reading K: reuse it for P
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) Ps[(4 * i + a) * kPaPs + j + 16 * b] = sc[a][b];
        __syncthreads();
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int d = 0; d < 8; ++d) o[a][d] *= alpha[a];
        const int tn = min(kPaKeys, last - t0 + 1);
        for (int t = 0; t < tn; t += 4) {
            float4 pa[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) pa[a] = *reinterpret_cast<const float4*>(Ps + (4 * i + a) * kPaPs + t);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float4 v0 = *reinterpret_cast<const float4*>(Vs + (t + u) * 128 + 4 * j);
                const float4 v1 = *reinterpret_cast<const float4*>(Vs + (t + u) * 128 + 64 + 4 * j);
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float p = u == 0 ? pa[a].x : u == 1 ? pa[a].y : u == 2 ? pa[a].z : pa[a].w;
                    o[a][0] = fmaf(p, v0.x, o[a][0]);
                    o[a][1] = fmaf(p, v0.y, o[a][1]);
                    o[a][2] = fmaf(p, v0.z, o[a][2]);
                    o[a][3] = fmaf(p, v0.w, o[a][3]);
                    o[a][4] = fmaf(p, v1.x, o[a][4]);
                    o[a][5] = fmaf(p, v1.y, o[a][5]);
                    o[a][6] = fmaf(p, v1.z, o[a][6]);
                    o[a][7] = fmaf(p, v1.w, o[a][7]);
                }
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        if (rpos[a] < 0) continue;
        const int r = 4 * i + a;
        const int sq = qlo + r / group, head = kvh * group + r % group;
        const float inv = 1.0f / l[a];
        float* dst = out + (size_t)sq * Hq + head * hd;
        *reinterpret_cast<float4*>(dst + 4 * j) =
            make_float4(o[a][0] * inv, o[a][1] * inv, o[a][2] * inv, o[a][3] * inv);
        *reinterpret_cast<float4*>(dst + 64 + 4 * j) =
            make_float4(o[a][4] * inv, o[a][5] * inv, o[a][6] * inv, o[a][7] * inv);
    }
}

tvb_status pf_attention(const float* q, const float* kcache, const float* vcache, int S, int pos0, int nh, int nkv,
                        int hd, float scale, float* out, cudaStream_t st) {
    TVB_REQUIRE(q && kcache && vcache && out && S > 0 && pos0 >= 0, "prefill attention: bad arguments");
    TVB_REQUIRE(hd == 128, "prefill attention: head_dim %d (only 128 is built)", hd);
    TVB_REQUIRE(nh > 0 && nkv > 0 && nh % nkv == 0 && kPaRows % (nh / nkv) == 0,
                "prefill attention: %d query heads per kv head must divide %d", nkv ? nh / nkv : 0, kPaRows);
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    std::call_once(once, [] {
        err = cudaFuncSetAttribute(pf_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPaSmem);
    });
    if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(pf_attn_kernel)");
    const int bq = kPaRows / (nh / nkv);
    const dim3 grid((unsigned)nkv, (unsigned)((S + bq - 1) / bq));
    pf_attn_kernel<<<grid, kPaThreads, kPaSmem, st>>>(q, kcache, vcache, S, pos0, nh, nkv, scale, out);
    return check_launch("pf_attn_kernel");
}

}  // namespace tvb
