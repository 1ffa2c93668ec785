// Load-time merge with the LoRA delta on the tensor cores (tvb_merge_batch_tc).
//
//   merged[n][k] = scale * map(code[n][k]) + (sum_j B[n][j] * A[j][k]) * (alpha / r)
//
// as in apply_lora (src/model.cpp:180-258), F16 output by truncation
// (tensor.cpp:33-57).  The rank-r contraction runs as tcgen05.mma
// (kind::f16, F32 accumulation in TMEM): B and A^T are split once per tensor
// into F16 hi + lo planes with power-of-two exponents per row of B and per
// column of A (largest magnitude of each in [2^14, 2^15)), and three MMAs per
// 16-wide k-step (hi.hi + hi.lo + lo.hi) give the delta to ~2^-21 of its
// largest term.  The F16 results are within one unit in the last place of the
// reference's sequential F32 sum (usually identical); tvb_merge_batch keeps the
// bit-exact CUDA-core path for F32, INT8 and ranks above 64.
//
// One CTA per 128-row stripe of a tensor: the stripe's B rows (hi, lo) stay in
// shared memory, the A^T column tiles (256 columns, hi, lo) stream through a
// double buffer with the tile's I2_S codes and column exponents, the MMAs of
// tile t run while the epilogue of tile t - 1 (I2_S unpack, scale, F16 cast)
// reads the other half of a 512-column TMEM accumulator and hands 32 x 32
// boxes to TMA stores.
#include "common.cuh"
#include "prefill.h"
#include "tcgen05.cuh"

#include <algorithm>

namespace tvb {

constexpr int kMtRows = 128;                  // W rows per stripe (MMA M)
constexpr int kMtCols = 256;                  // W columns per tile (MMA N)
constexpr int kMtRank = 64;                   // padded rank: one 128-byte swizzle row of F16
constexpr int kMtThreads = 512;
constexpr int kMtMaxDescs = 192;
constexpr int kMtAop = kMtRows * 128;         // bytes per plane of the stripe's B rows
constexpr int kMtBop = kMtCols * 128;         // bytes per plane of an A^T tile
// the column exponents rotate over 3 tiles: tile t + 1 is staged while the
// epilogue of tile t - 1 still reads its own
// then one output box per warp: 32 rows x 32 F16 columns (64 bytes, 64-byte
// swizzle) written by the warp and stored by TMA
constexpr int kMtBox = 32 * 32 * 2;
constexpr int kMtOutOff = ((2 * kMtAop + 4 * kMtBop + 3 * kMtCols * 4 + kMtRows * 4 + 64 + 1023) / 1024) * 1024;
// then the I2_S codes of the stripe's rows for 3 tiles (rotating like the
// exponents): 128 rows x 2 blocks x 32 bytes each
constexpr int kMtCodes = kMtRows * 64;
constexpr int kMtCodeOff = kMtOutOff + (kMtThreads / 32) * kMtBox;
constexpr int kMtSmem = kMtCodeOff + 3 * kMtCodes + 1024;

struct MtDesc {
    const uint8_t* i2s;      // whole tensor's codes (row pitch ld / 4 bytes)
    const uint16_t* bh;      // [N][64] F16 hi of B * 2^-eb[n]
    const uint16_t* bl;
    const int* eb;           // [N]
    const uint16_t* ath;     // [K][64] F16 hi of A^T * 2^-ea[k]
    const uint16_t* atl;
    const float* fa;         // [K] 2^ea: A^T column k was stored scaled by 2^-ea[k]
    uint16_t* dst;           // [N][K] F16
    const float* A;          // LoRA A [r][ld] (whole tensor's columns)
    const float* B;          // LoRA B [N][r]
    float scale;             // I2_S per-tensor scale
    float sf;                // alpha / r
    int K, N, r, k0, ld;
    int a_row0;              // first row of ath / atl in the launch's plane maps
};

struct MtBatch {
    MtDesc d[kMtMaxDescs];
    const CUtensorMap* omaps;   // [n] output maps (device memory): dst [N][K] F16, 32 x 32 boxes
    const CUtensorMap* amaps;   // [2] the A^T hi and lo planes of every tensor of the launch
                                // ([columns][64] F16, 256-row boxes, 128-byte swizzle)
    int cta_start[kMtMaxDescs + 1];   // merge CTAs (128-row stripes)
    int row_start[kMtMaxDescs + 1];   // prep warps (rows of B)
    int col_start[kMtMaxDescs + 1];   // prep threads (columns of A)
    int n;
};

// Descriptor owning global unit `u` of a start table.
__device__ __forceinline__ int mt_owner(const int* start, int n, int u) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (start[mid] <= u) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ int mt_find(const MtBatch& b, int cta) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (b.cta_start[mid] <= cta) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// Power-of-two exponent putting |m| in [2^14, 2^15) (0 for zero rows).
__device__ __forceinline__ int mt_exp(float m) {
    return (m > 0.f && isfinite(m)) ? max(ilogbf(m) - 14, -100) : 0;
}

// 2^e as a float (e within the normal range is built from its bits).
__device__ __forceinline__ float mt_pow2(int e) {
    return (e >= -126 && e <= 127) ? __int_as_float((e + 127) << 23) : ldexpf(1.0f, e);
}

__device__ __forceinline__ void mt_split(float v, float sc, __half& hi, __half& lo) {
    const float f = v * sc;
    hi = __float2half_rn(f);
    lo = __float2half_rn(f - __half2float(hi));
}

// B rows -> hi/lo planes: one warp per row (rank <= 64: lanes own j, j + 32).
__global__ void mt_prep_b(const __grid_constant__ MtBatch b) {
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int lo = mt_owner(b.row_start, b.n, gw);
    const MtDesc& d = b.d[lo];
    const int n = gw - b.row_start[lo];
    if (n < 0 || n >= d.N) return;
    const float* B = d.B;
    const float v0 = (lane < d.r) ? B[(size_t)n * d.r + lane] : 0.f;
    const float v1 = (lane + 32 < d.r) ? B[(size_t)n * d.r + lane + 32] : 0.f;
    const int e = mt_exp(warp_max(fmaxf(fabsf(v0), fabsf(v1))));
    const float sc = ldexpf(1.0f, -e);
    __half h0, l0, h1, l1;
    mt_split(v0, sc, h0, l0);
    mt_split(v1, sc, h1, l1);
    __half* bh = reinterpret_cast<__half*>(const_cast<uint16_t*>(d.bh)) + (size_t)n * kMtRank;
    __half* bl = reinterpret_cast<__half*>(const_cast<uint16_t*>(d.bl)) + (size_t)n * kMtRank;
    bh[lane] = h0;
    bh[lane + 32] = h1;
    bl[lane] = l0;
    bl[lane + 32] = l1;
    if (lane == 0) const_cast<int*>(d.eb)[n] = e;
}

// Columns [k0, k0 + K) of A [r][ld] -> A^T hi/lo planes: one thread per column.
__global__ void mt_prep_a(const __grid_constant__ MtBatch b) {
    const int gc = blockIdx.x * blockDim.x + threadIdx.x;
    const int lo = mt_owner(b.col_start, b.n, gc);
    const MtDesc& d = b.d[lo];
    const int k = gc - b.col_start[lo];
    if (k < 0 || k >= d.K) return;
    const float* A = d.A;
    float m = 0.f;
    for (int j = 0; j < d.r; ++j) m = fmaxf(m, fabsf(A[(size_t)j * d.ld + d.k0 + k]));
    const int e = mt_exp(m);
    const float sc = ldexpf(1.0f, -e);
    uint4* th = reinterpret_cast<uint4*>(const_cast<uint16_t*>(d.ath) + (size_t)k * kMtRank);
    uint4* tl = reinterpret_cast<uint4*>(const_cast<uint16_t*>(d.atl) + (size_t)k * kMtRank);
    for (int c = 0; c < kMtRank / 8; ++c) {
        __half h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int j = c * 8 + i;
            mt_split(j < d.r ? A[(size_t)j * d.ld + d.k0 + k] : 0.f, sc, h[i], l[i]);
        }
        th[c] = *reinterpret_cast<const uint4*>(h);
        tl[c] = *reinterpret_cast<const uint4*>(l);
    }
    const_cast<float*>(d.fa)[k] = mt_pow2(e);
}

// Packed F32 pairs (one instruction for two IEEE-rounded lanes).
__device__ __forceinline__ float2 mt_mul2(float2 a, float2 b) {
    uint64_t d;
    const uint64_t ua = (uint64_t)__float_as_uint(a.x) | ((uint64_t)__float_as_uint(a.y) << 32);
    const uint64_t ub = (uint64_t)__float_as_uint(b.x) | ((uint64_t)__float_as_uint(b.y) << 32);
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(ua), "l"(ub));
    return make_float2(__uint_as_float((uint32_t)d), __uint_as_float((uint32_t)(d >> 32)));
}
__device__ __forceinline__ float2 mt_fma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    const uint64_t ua = (uint64_t)__float_as_uint(a.x) | ((uint64_t)__float_as_uint(a.y) << 32);
    const uint64_t ub = (uint64_t)__float_as_uint(b.x) | ((uint64_t)__float_as_uint(b.y) << 32);
    const uint64_t uc = (uint64_t)__float_as_uint(c.x) | ((uint64_t)__float_as_uint(c.y) << 32);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(ua), "l"(ub), "l"(uc));
    return make_float2(__uint_as_float((uint32_t)d), __uint_as_float((uint32_t)(d >> 32)));
}

__device__ __forceinline__ void mt_fail(unsigned* status) {
    if (status) atomicOr(status, kStatusTimeout);
}

__global__ void __launch_bounds__(kMtThreads, 1)
merge_tc_kernel(const __grid_constant__ MtBatch b, unsigned* status) {
    extern __shared__ unsigned char mt_smem_raw[];
    const uint32_t raw = smem_u32(mt_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = mt_smem_raw + (base - raw);
    const uint32_t a_hi = base, a_lo = base + kMtAop;
    const uint32_t b_op = base + 2 * kMtAop;                    // [buf][plane] tiles of kMtBop
    float* fa_s = reinterpret_cast<float*>(smem + 2 * kMtAop + 4 * kMtBop);   // [3][256] 2^ea, tile % 3
    int* eb_s = reinterpret_cast<int*>(fa_s + 3 * kMtCols);                   // [128]
    uint64_t* mbar = reinterpret_cast<uint64_t*>(eb_s + kMtRows);        // [2] MMA done, [2] A^T tile landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int di = mt_find(b, blockIdx.x);
    const MtDesc& d = b.d[di];
    const int row0 = (blockIdx.x - b.cta_start[di]) * kMtRows;

    // the stripe's B rows (hi, lo) and their exponents
    for (int idx = tid; idx < kMtRows * 8; idx += kMtThreads) {
        const int r = idx >> 3, c = idx & 7;
        uint4 h = make_uint4(0u, 0u, 0u, 0u), l = h;
        if (row0 + r < d.N) {
            h = *reinterpret_cast<const uint4*>(d.bh + (size_t)(row0 + r) * kMtRank + c * 8);
            l = *reinterpret_cast<const uint4*>(d.bl + (size_t)(row0 + r) * kMtRank + c * 8);
        }
        *reinterpret_cast<uint4*>(smem + sw128_offset(r, c)) = h;
        *reinterpret_cast<uint4*>(smem + kMtAop + sw128_offset(r, c)) = l;
    }
    for (int r = tid; r < kMtRows; r += kMtThreads) eb_s[r] = row0 + r < d.N ? d.eb[row0 + r] : 0;
    if (tid == 0) {
        for (int i = 0; i < 4; ++i) mbar_init(&mbar[i], 1);
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    fence_proxy_async_smem_cta();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int ntiles = (d.K + kMtCols - 1) / kMtCols;
    const int q = warp & 3, cq = warp >> 2;          // TMEM lane quarter, column quarter (64)
    const uint32_t obox = base + (uint32_t)(kMtOutOff + warp * kMtBox);
    // the output map was written into device memory by a copy before this
    // launch: acquire it for the tensor-map proxy before the first store
    if (lane == 0)
        asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(b.omaps + di) : "memory");
    if (tid == 0)
        for (int i = 0; i < 2; ++i)
            asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(b.amaps + i) : "memory");
    const int rloc = 32 * q + lane;
    const int src_blocks = d.ld >> 7, blk0 = d.k0 >> 7;
    // A^T tile t (256 columns, hi and lo) into buffer `buf`: two TMA loads
    // (128-byte swizzle, the layout the MMA descriptors expect) completing on
    // mbar[2 + buf].  Rows past this tensor's K belong to the next tensor of
    // the launch (zeros past the last): they only reach output columns past K,
    // which the tile's stores clip.  The tile's codes and column exponents go
    // into rotating slot t % 3 by asynchronous 16-byte copies, zero past N / K.
    auto load_tile = [&](int t, int buf) {
        if (tid == 0) {
            const uint32_t dst = b_op + (uint32_t)(2 * buf) * kMtBop;
            mbar_expect_tx(&mbar[2 + buf], 2u * kMtBop);
            tma_load_2d(dst, b.amaps, 0, d.a_row0 + t * kMtCols, &mbar[2 + buf]);
            tma_load_2d(dst + kMtBop, b.amaps + 1, 0, d.a_row0 + t * kMtCols, &mbar[2 + buf]);
        }
        // the stripe's I2_S codes of these columns (two 32-byte blocks a row),
        // zero past N and K
        for (int idx = tid; idx < kMtRows * 4; idx += kMtThreads) {
            const int r = idx >> 2, j = idx & 3, blk = 2 * t + (j >> 1);
            const bool in = row0 + r < d.N && blk * 128 < d.K;
            const uint8_t* src = d.i2s + (in ? ((size_t)(row0 + r) * src_blocks + blk0 + blk) * 32 + (j & 1) * 16 : 0);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                             base + (uint32_t)(kMtCodeOff + (t % 3) * kMtCodes + r * 64 + j * 16)),
                         "l"(src), "r"(in ? 16u : 0u)
                         : "memory");
        }
        // the columns' 2^ea ride in the same group (16-byte copies, zero past K)
        for (int r4 = tid; r4 < kMtCols / 4; r4 += kMtThreads) {
            const int col = t * kMtCols + 4 * r4;
            const bool in = col < d.K;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                             smem_u32(fa_s + (t % 3) * kMtCols + 4 * r4)),
                         "l"(d.fa + (in ? col : 0)), "r"(in ? 16u : 0u)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    bool ok = true;
    load_tile(0, 0);
    for (int t = 0; t <= ntiles; ++t) {
        // MMA(t - 1) done: its A^T buffer is free for tile t + 1, its accumulator ready
        if (t > 0 && ok && !mbar_wait_bounded(&mbar[(t - 1) & 1], (uint32_t)(((t - 1) >> 1) & 1))) {
            ok = false;
            mt_fail(status);
        }
        if (t + 1 < ntiles) load_tile(t + 1, (t + 1) & 1);
        if (t < ntiles) {
            const int buf = t & 1;
            if (t + 1 < ntiles) asm volatile("cp.async.wait_group 1;" ::: "memory");
            else asm volatile("cp.async.wait_group 0;" ::: "memory");
            fence_proxy_async_smem_cta();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0 && ok && !mbar_wait_bounded(&mbar[2 + buf], (uint32_t)((t >> 1) & 1))) {
                ok = false;
                mt_fail(status);
            }
            if (tid == 0 && ok) {
                constexpr uint32_t idesc = umma_idesc_f16(kMtRows, kMtCols);
                const uint32_t dcol = tmem + (uint32_t)(buf * kMtCols);
                const uint32_t bh_s = b_op + (uint32_t)(2 * buf) * kMtBop, bl_s = bh_s + kMtBop;
#pragma unroll
                for (int kk = 0; kk < kMtRank / 16; ++kk) {
                    const uint64_t ah = sw128_desc(a_hi + kk * 32), al = sw128_desc(a_lo + kk * 32);
                    const uint64_t bh = sw128_desc(bh_s + kk * 32), bl = sw128_desc(bl_s + kk * 32);
                    tc_mma(dcol, ah, bh, idesc, kk ? 1u : 0u);
                    tc_mma(dcol, ah, bl, idesc, 1u);
                    tc_mma(dcol, al, bh, idesc, 1u);
                }
                tc_commit(&mbar[buf]);
            }
        }
        if (t > 0) {
            const int u = t - 1, ubuf = u & 1;
            const int colh = u * kMtCols + cq * 64;      // first of this thread's 64 columns
            const bool rowok = ok && colh < d.K;   // (uniform over the warp)
            // their I2_S codes: the 32-byte block of this row that holds them
            const uint4* cw = reinterpret_cast<const uint4*>(smem + kMtCodeOff + (u % 3) * kMtCodes + rloc * 64 +
                                                             (cq >> 1) * 32);
            const uint4 w0 = cw[0], w1 = cw[1];
            const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            // per row: alpha / r times 2^eb (both exact powers-of-two scalings of
            // the delta, applied as (acc * 2^ea) * (sf * 2^eb): one rounding, as
            // the reference's delta * sf)
            const float g = d.sf * mt_pow2(eb_s[rloc]);
            const float4* fa4 = reinterpret_cast<const float4*>(fa_s + (u % 3) * kMtCols + cq * 64);
            // bits of map2bit(code) * scale (tensor.cpp:1020): code 0 -> -scale,
            // 2 -> +scale (the sign bit flipped by the code's bit 1), 1 and 3 -> +0
            const uint32_t sn_bits = __float_as_uint(-d.scale);
            for (int c = 0; c < 2; ++c) {
                __syncwarp();
                uint32_t acc[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(ubuf * kMtCols + cq * 64 + c * 32), acc);
                tmem_wait_ld();
                if (!rowok) continue;
                // column 32 * slot + j of the block: byte j, bits shift + 1 .. shift
                const int shift = 6 - 2 * (((colh & 127) >> 5) + c);
                // merged = map(code) * scale + acc * 2^ea * (alpha / r) * 2^eb; the
                // column and row factors are powers of two apart from alpha / r,
                // so 2^ea * g is exact and one fused multiply-add does the rest
                // (one rounding where the exact merge has two: the F16 result
                // stays within one unit in the last place)
                float mv[32];
                float mx = 0.f;
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 fa = fa4[c * 8 + j4];
                    // column j = 4 j4 + i: its code is bits [8 i + 1, 8 i] of cw
                    const uint32_t cw = words[j4] >> shift;
                    float bv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t odd;
                        asm("bfe.s32 %0, %1, %2, 1;" : "=r"(odd) : "r"(cw), "r"(8 * i));   // -1 for codes 1, 3
                        bv[i] = __uint_as_float((sn_bits ^ ((cw << (30 - 8 * i)) & 0x80000000u)) & ~odd);
                    }
                    const float2 gg = make_float2(g, g);
                    const float2 m01 = mt_fma2(make_float2(__uint_as_float(acc[4 * j4]), __uint_as_float(acc[4 * j4 + 1])),
                                               mt_mul2(make_float2(fa.x, fa.y), gg), make_float2(bv[0], bv[1]));
                    const float2 m23 = mt_fma2(make_float2(__uint_as_float(acc[4 * j4 + 2]), __uint_as_float(acc[4 * j4 + 3])),
                                               mt_mul2(make_float2(fa.z, fa.w), gg), make_float2(bv[2], bv[3]));
                    mv[4 * j4] = m01.x;
                    mv[4 * j4 + 1] = m01.y;
                    mv[4 * j4 + 2] = m23.x;
                    mv[4 * j4 + 3] = m23.y;
                    mx = fmaxf(fmaxf(mx, fmaxf(fabsf(m01.x), fabsf(m01.y))), fmaxf(fabsf(m23.x), fabsf(m23.y)));
                }
                uint32_t packed[16];
                if (mx < 65536.0f) {
                    // round toward zero = the reference's truncation in this range
#pragma unroll
                    for (int t = 0; t < 16; ++t)
                        asm("cvt.rz.f16x2.f32 %0, %1, %2;" : "=r"(packed[t]) : "f"(mv[2 * t + 1]), "f"(mv[2 * t]));
                } else {
#pragma unroll
                    for (int t = 0; t < 16; ++t)
                        packed[t] = (uint32_t)f32_to_f16_trunc(mv[2 * t]) |
                                    ((uint32_t)f32_to_f16_trunc(mv[2 * t + 1]) << 16);
                }
                // the warp's 32 rows x these 32 columns as one box: lane = row,
                // 64 bytes in 16-byte chunks at their 64-byte-swizzled places
                // (conflict-free per 8-lane phase); then one TMA store, which
                // clips rows past N
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int v = 0; v < 4; ++v)
                    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(
                                     obox + (uint32_t)(lane * 64 + ((v ^ ((lane >> 1) & 3)) * 16))),
                                 "r"(packed[4 * v]), "r"(packed[4 * v + 1]), "r"(packed[4 * v + 2]),
                                 "r"(packed[4 * v + 3])
                                 : "memory");
                fence_proxy_async_smem_cta();
                __syncwarp();
                if (lane == 0) {
                    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                                     reinterpret_cast<uint64_t>(b.omaps + di)),
                                 "r"(colh + c * 32), "r"(row0 + 32 * q), "r"(obox)
                                 : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            tc_fence_before();
        }
        __syncthreads();
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // every output box written
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Per-row INT8 of merged F16 rows (the reference's quantisation of the F16
// weights, tensor.cpp absmax per row): one warp per row, a max pass then a
// code pass, 16 elements per lane step (K % 128 == 0).
struct MtQuant {
    const uint16_t* f16[kMtMaxDescs];
    int8_t* q[kMtMaxDescs];
    float* scales[kMtMaxDescs];
    int K[kMtMaxDescs];
    int row_start[kMtMaxDescs + 1];
    int n;
};

__global__ void __launch_bounds__(256) mt_quant_kernel(const __grid_constant__ MtQuant b) {
    const int grow = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int i = mt_owner(b.row_start, b.n, grow);
    const int row = grow - b.row_start[i];
    if (row < 0 || grow >= b.row_start[b.n]) return;
    const int K = b.K[i];
    const uint16_t* src = b.f16[i] + (size_t)row * K;
    uint32_t m = 0;
    for (int e = lane * 8; e < K; e += 32 * 8) {
        const uint4 h = *reinterpret_cast<const uint4*>(src + e);
        const uint32_t w[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) m = max(m, max(w[t] & 0x7FFFu, (w[t] >> 16) & 0x7FFFu));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    float mx = __half2float(__ushort_as_half((uint16_t)m));
    if (mx == 0.0f) mx = 1.0f;
    const float s = __fdiv_rn(mx, 127.0f);
    if (lane == 0) b.scales[i][row] = s;
    int8_t* out = b.q[i] + (size_t)row * K;
    for (int e = lane * 16; e < K; e += 32 * 16) {
        const uint4 hv = *reinterpret_cast<const uint4*>(src + e);
        const uint4 hw = *reinterpret_cast<const uint4*>(src + e + 8);
        const uint32_t hs[8] = {hv.x, hv.y, hv.z, hv.w, hw.x, hw.y, hw.z, hw.w};
        uint32_t words[4];
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
            uint32_t acc = 0;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const uint32_t h2 = hs[2 * qd + t];
                const float lo_v = __half2float(__ushort_as_half((uint16_t)(h2 & 0xFFFFu)));
                const float hi_v = __half2float(__ushort_as_half((uint16_t)(h2 >> 16)));
                acc |= ((uint32_t)(uint8_t)int8_code(lo_v, s)) << (16 * t);
                acc |= ((uint32_t)(uint8_t)int8_code(hi_v, s)) << (16 * t + 8);
            }
            words[qd] = acc;
        }
        *reinterpret_cast<uint4*>(out + e) = make_uint4(words[0], words[1], words[2], words[3]);
    }
}

static tvb_status mt_prepare() {
    static cudaError_t err = cudaErrorNotReady;
    if (err == cudaErrorNotReady) {
        err = cudaFuncSetAttribute(merge_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMtSmem);
        // keep the stream-ordered pool's memory between calls (the workspace is
        // a few hundred MB for a whole model and would otherwise be unmapped
        // and mapped again at every synchronisation)
        int dev = 0;
        cudaMemPool_t pool;
        if (err == cudaSuccess && cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
            uint64_t keep = ~0ull;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        }
    }
    if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(merge_tc_kernel)");
    return TVB_OK;
}

tvb_status merge_exact(const tvb_merge_desc* descs, int n, tvb_dtype out, cudaStream_t st);

tvb_status merge_tc(const tvb_merge_desc* descs, int n, tvb_dtype out, cudaStream_t st);

// Per-row INT8 through the tensor cores: groups of tensors are merged to F16
// into a workspace (at most kMtI8Workspace bytes a group) and quantised per
// row from there.  The codes are the reference's quantisation of these F16
// weights, which are within one F16 unit in the last place of its own.
constexpr size_t kMtI8Workspace = 512ull << 20;

static tvb_status merge_tc_i8(const tvb_merge_desc* descs, int n, cudaStream_t st) {
    size_t need = 0, total = 0;
    for (int i = 0; i < n; ++i) {
        TVB_REQUIRE(descs[i].row_scales, "merge_tc: descriptor %d: per-row INT8 needs row_scales", i);
        const size_t b16 = ((size_t)descs[i].N * descs[i].K * 2 + 255) / 256 * 256;
        need = std::max(need, b16);
        total += b16;
    }
    const size_t ws_bytes = std::max(need, std::min(kMtI8Workspace, total));
    unsigned char* ws = nullptr;
    TVB_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&ws), ws_bytes, st));
    static thread_local tvb_merge_desc f16d[kMtMaxDescs];
    static thread_local MtQuant qb;
    tvb_status result = TVB_OK;
    int i = 0;
    while (i < n && result == TVB_OK) {
        size_t used = 0;
        int cnt = 0, rows = 0;
        while (i + cnt < n && cnt < kMtMaxDescs) {
            const tvb_merge_desc& s = descs[i + cnt];
            const size_t b16 = ((size_t)s.N * s.K * 2 + 255) / 256 * 256;
            if (cnt > 0 && used + b16 > ws_bytes) break;
            f16d[cnt] = s;
            f16d[cnt].dst = ws + used;
            f16d[cnt].row_scales = nullptr;
            qb.f16[cnt] = reinterpret_cast<const uint16_t*>(ws + used);
            qb.q[cnt] = static_cast<int8_t*>(s.dst);
            qb.scales[cnt] = s.row_scales;
            qb.K[cnt] = s.K;
            qb.row_start[cnt] = rows;
            rows += s.N;
            used += b16;
            ++cnt;
        }
        qb.row_start[cnt] = rows;
        qb.n = cnt;
        result = merge_tc(f16d, cnt, TVB_F16, st);
        if (result != TVB_OK) break;
        mt_quant_kernel<<<(rows + 7) / 8, 256, 0, st>>>(qb);
        result = check_launch("mt_quant_kernel");
        i += cnt;
    }
    const cudaError_t e = cudaFreeAsync(ws, st);
    if (result == TVB_OK && e != cudaSuccess) result = cuda_error(e, "cudaFreeAsync");
    return result;
}

tvb_status merge_tc(const tvb_merge_desc* descs, int n, tvb_dtype out, cudaStream_t st) {
    if (n <= 0) return TVB_OK;
    TVB_REQUIRE(descs, "merge_tc: descs is NULL");
    bool exact = out != TVB_F16 && out != TVB_I8_ROW;
    for (int i = 0; i < n && !exact; ++i) exact = descs[i].r > kMtRank;
    if (exact) return merge_exact(descs, n, out, st);   // F32 / per-tensor INT8 / rank > 64: bit-exact path
    if (out == TVB_I8_ROW) return merge_tc_i8(descs, n, st);
    for (int i = 0; i < n; ++i) {
        const tvb_merge_desc& s = descs[i];
        const int ld = s.ld ? s.ld : s.K;
        TVB_REQUIRE(s.i2s && s.dst && s.K > 0 && s.N > 0 && s.K % 128 == 0, "merge_tc: descriptor %d", i);
        TVB_REQUIRE(s.r >= 0 && (s.r == 0 || (s.A && s.B)), "merge_tc: rank %d needs A and B", s.r);
        TVB_REQUIRE(s.k0 >= 0 && s.k0 % 128 == 0 && ld % 128 == 0 && s.k0 + s.K <= ld,
                    "merge_tc: column slice [%d, %d) of %d columns", s.k0, s.k0 + s.K, ld);
        TVB_REQUIRE((reinterpret_cast<uintptr_t>(s.dst) & 15) == 0 && (reinterpret_cast<uintptr_t>(s.i2s) & 15) == 0,
                    "merge_tc: dst and i2s must be 16-byte aligned");
    }
    TVB_TRY(mt_prepare());
    static thread_local MtBatch b;
    for (int base = 0; base < n; base += kMtMaxDescs) {
        const int cnt = std::min(kMtMaxDescs, n - base);
        // workspace: prepared planes and exponents of every tensor of this launch
        size_t rows = 0, cols = 0;
        for (int i = 0; i < cnt; ++i) {
            rows += (size_t)descs[base + i].N;
            cols += (size_t)descs[base + i].K;
        }
        // (output tensor maps, then the two A^T plane maps, first: 128-byte aligned)
        const size_t map_bytes = (size_t)(cnt + 2) * sizeof(CUtensorMap);
        const size_t bytes = map_bytes + 2 * (rows + cols) * kMtRank * 2 + (rows + cols) * 4 + 256;
        unsigned char* ws = nullptr;
        TVB_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&ws), bytes, st));
        static thread_local CUtensorMap omaps[kMtMaxDescs + 2];
        for (int i = 0; i < cnt; ++i) {
            const tvb_merge_desc& sd = descs[base + i];
            const uint64_t dims[2] = {(uint64_t)sd.K, (uint64_t)sd.N};
            const uint64_t strides[1] = {(uint64_t)sd.K * 2};
            const uint32_t box[2] = {32u, 32u};
            tvb_status es = encode_f16_tiled(&omaps[i], sd.dst, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
            if (es != TVB_OK) {
                cudaFreeAsync(ws, st);
                return es;
            }
        }
        uint16_t* bh = reinterpret_cast<uint16_t*>(ws + map_bytes);
        uint16_t* bl = bh + rows * kMtRank;
        uint16_t* ah = bl + rows * kMtRank;
        uint16_t* al = ah + cols * kMtRank;
        for (int i = 0; i < 2; ++i) {
            const uint64_t dims[2] = {(uint64_t)kMtRank, (uint64_t)cols};
            const uint64_t strides[1] = {(uint64_t)kMtRank * 2};
            const uint32_t box[2] = {(uint32_t)kMtRank, (uint32_t)kMtCols};
            tvb_status es = encode_f16_tiled(&omaps[cnt + i], i ? al : ah, 2, dims, strides, box,
                                             CU_TENSOR_MAP_SWIZZLE_128B);
            if (es != TVB_OK) {
                cudaFreeAsync(ws, st);
                return es;
            }
        }
        {
            const cudaError_t ce = cudaMemcpyAsync(ws, omaps, map_bytes, cudaMemcpyHostToDevice, st);
            if (ce != cudaSuccess) {
                cudaFreeAsync(ws, st);
                return cuda_error(ce, "cudaMemcpyAsync(merge output maps)");
            }
        }
        b.omaps = reinterpret_cast<const CUtensorMap*>(ws);
        b.amaps = b.omaps + cnt;
        int* eb = reinterpret_cast<int*>(al + cols * kMtRank);
        // (16-byte aligned: the kernel copies it in 16-byte pieces)
        float* fa = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(eb + rows) + 15) & ~(uintptr_t)15);
        size_t ro = 0, co = 0;
        int ctas = 0, rwarps = 0, cthreads = 0;
        for (int i = 0; i < cnt; ++i) {
            const tvb_merge_desc& s = descs[base + i];
            MtDesc& d = b.d[i];
            d.i2s = s.i2s;
            d.bh = bh + ro * kMtRank;
            d.bl = bl + ro * kMtRank;
            d.eb = eb + ro;
            d.ath = ah + co * kMtRank;
            d.atl = al + co * kMtRank;
            d.fa = fa + co;
            d.dst = static_cast<uint16_t*>(s.dst);
            d.A = s.r ? s.A : nullptr;
            d.B = s.r ? s.B : nullptr;
            d.scale = s.scale;
            d.sf = s.r ? s.alpha / (float)s.r : 0.0f;
            d.K = s.K;
            d.N = s.N;
            d.r = s.r;
            d.k0 = s.k0;
            d.ld = s.ld ? s.ld : s.K;
            d.a_row0 = (int)co;
            b.cta_start[i] = ctas;
            b.row_start[i] = rwarps;
            b.col_start[i] = cthreads;
            ctas += (s.N + kMtRows - 1) / kMtRows;
            rwarps += s.N;
            cthreads += s.K;
            ro += (size_t)s.N;
            co += (size_t)s.K;
        }
        b.cta_start[cnt] = ctas;
        b.row_start[cnt] = rwarps;
        b.col_start[cnt] = cthreads;
        b.n = cnt;
        mt_prep_b<<<(rwarps + 7) / 8, 256, 0, st>>>(b);
        tvb_status s = check_launch("mt_prep_b");
        if (s == TVB_OK) {
            mt_prep_a<<<(cthreads + 255) / 256, 256, 0, st>>>(b);
            s = check_launch("mt_prep_a");
        }
        if (s == TVB_OK) {
            merge_tc_kernel<<<ctas, kMtThreads, kMtSmem, st>>>(b, nullptr);
            s = check_launch("merge_tc_kernel");
        }
        cudaFreeAsync(ws, st);
        if (s != TVB_OK) return s;
    }
    return TVB_OK;
}

}  // namespace tvb

extern "C" tvb_status tvb_merge_batch_tc(const tvb_merge_desc* descs, int n, tvb_dtype out, void* stream) {
    return tvb::merge_tc(descs, n, out, tvb::as_stream(stream));
}
