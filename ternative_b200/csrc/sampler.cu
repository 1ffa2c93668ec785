// The token sampler on the device (sample_token, src/sampler.cpp:11-148) for B
// rows of logits, so a batched decode step need not copy 128k logits per row
// to the host.  One 8-CTA cluster per row (sample_cluster_kernel; rows longer
// than 196,608 entries: one CTA, sample_kernel) runs the reference's steps in
// its order and arithmetic:
//
//   1. logits / temperature (when temperature > 0 and != 1)
//   2. repetition penalty: each distinct seen token's value / penalty once
//   3. softmax: exp(v - max) in F32, the sum in F64, p = (float)(e / sum)
//   4. top-k: keep the k largest (p, index) pairs (ties: the larger index)
//   5. top-p: of the kept p > 0, sorted by (p, index) descending, the shortest
//      prefix whose F32 running sum reaches top_p
//   6. renormalise (F64 sum, F32 result); nothing left -> argmax of the logits
//   7. F32 running sum in index order; the first index whose sum >= u
//
// The uniform draw u of step 7 is the caller's (the reference draws it from
// its own mt19937).  Sums the reference takes in index order are taken as
// trees here: the F64 sums differ from it only far below F32 resolution, and
// the step-7 running sum runs sequentially in index order over the entries
// that can be nonzero, as the reference's.  The cluster kernel's top-p works
// on at most 1024 candidates (1 <= top_k <= 1024); top-p with top_k 0 (the
// whole vocabulary) or above 1024 runs on sample_kernel, which walks the
// sorted keys 1024 at a time.
#include <cuda_runtime.h>

#include <cfloat>

#include <cooperative_groups.h>

#include "sampler.h"

namespace tvb {

namespace cg = cooperative_groups;

constexpr int kSampThreads = 1024;
constexpr int kSampCand = 1024;
constexpr int kSampPer = 4;                         // entries per thread in a step-7 tile
constexpr int kSampTile = kSampThreads * kSampPer;
constexpr int kMaxLogprobs = kMaxLogprobsHost;

struct SampArgs {
    const float* logits;
    int vocab, ld;
    float temperature, penalty, top_p;
    int top_k;
    const int* seen;      // [B][max_seen]
    const int* n_seen;    // [B]
    int max_seen;
    const float* u;       // [B]
    int* out;             // [B]
    float* work;          // [B][vocab] probabilities
    unsigned* bits;       // [B][vocab / 32 + 1] penalty marks
};

__device__ __forceinline__ unsigned long long samp_key(float p, int i) {
    return ((unsigned long long)__float_as_uint(p) << 32) | (unsigned)i;   // p >= 0: bit order = value order
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = red[lane];   // 32 warps
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

// One radix-select step, run by warp 0: the bin d of the need-th largest key
// among those counted in hist[256] -- the first bin, from 255 down, whose
// running count reaches need (bin 0 if none does) -- and the rank left within
// it.  Lane l owns bins 255 - 8l .. 248 - 8l; a warp scan replaces the walk
// over the bins.
__device__ __forceinline__ void radix_pick(const unsigned* hist, int need, int* keep, int* left) {
    const int lane = threadIdx.x & 31;
    unsigned c[8], tot = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        tot += c[j];
    }
    unsigned incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const unsigned excl = incl - tot;
    const unsigned un = (unsigned)need;
    // bins 255 .. 1 only: bin 0 takes whatever is left
    const unsigned last = lane == 31 ? incl - c[7] : incl;
    const unsigned bal = __ballot_sync(0xffffffffu, excl < un && un <= last);
    if (bal == 0u) {
        if (lane == 31) {
            *keep = 0;
            *left = need - (int)(incl - c[7]);
        }
        return;
    }
    if (lane == __ffs(bal) - 1) {
        unsigned run = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (run + c[j] >= un) {
                *keep = 255 - 8 * lane - j;
                *left = need - (int)run;
                break;
            }
            run += c[j];
        }
    }
}

// The need-th largest of the keys key(i), i in [0, V), by an 8-bit radix
// select (1 <= need <= the number of nonzero keys); block-wide, all threads
// return it.
template <class Key>
__device__ __forceinline__ unsigned long long block_radix_kth(Key&& key, int V, int need, unsigned* hist,
                                                              int* s_keep, int* s_count) {
    const int tid = threadIdx.x;
    unsigned long long prefix = 0ull, mask = 0ull;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kSampThreads) hist[i] = 0u;
        __syncthreads();
        // warp-aggregated counts: the probabilities crowd into few bins
        for (int base = 0; base < V; base += kSampThreads) {
            const int i = base + tid;
            const unsigned long long k = i < V ? key(i) : 0ull;
            const bool hit = i < V && (k & mask) == prefix;
            const unsigned act = __ballot_sync(0xffffffffu, hit);
            if (hit) {
                const unsigned bin = (unsigned)(k >> shift) & 255u;
                const unsigned peers = __match_any_sync(act, bin);
                if ((tid & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], (unsigned)__popc(peers));
            }
        }
        __syncthreads();
        if (tid < 32) radix_pick(hist, need, s_keep, s_count);
        __syncthreads();
        prefix |= (unsigned long long)*s_keep << shift;
        mask |= 255ull << shift;
        need = *s_count;
        __syncthreads();
    }
    return prefix;
}

__global__ void __launch_bounds__(kSampThreads) sample_kernel(const __grid_constant__ SampArgs a) {
    const int b = blockIdx.x, tid = threadIdx.x, V = a.vocab;
    const float* lg = a.logits + (size_t)b * a.ld;
    float* p = a.work + (size_t)b * V;
    unsigned* bits = a.bits + (size_t)b * (V / 32 + 1);
    __shared__ double red_d[32];
    __shared__ float red_f[32];
    __shared__ unsigned long long red_k[32];
    __shared__ unsigned long long cand[kSampCand];
    __shared__ int s_count, s_keep, s_token;
    __shared__ unsigned hist[256];
    __shared__ float tile_v[kSampTile];
    __shared__ int tile_i[kSampTile];
    __shared__ int warp_cnt[32];

    // 1-2. temperature, then the repetition penalty on first occurrences
    const bool temp = a.temperature > 0.0f && a.temperature != 1.0f;
    for (int i = tid; i < V; i += kSampThreads) p[i] = temp ? lg[i] / a.temperature : lg[i];
    for (int i = tid; i < V / 32 + 1; i += kSampThreads) bits[i] = 0u;
    __syncthreads();
    if (a.penalty > 1.0f) {
        const int n = min(a.n_seen[b], a.max_seen);
        // distinct tokens only: the first thread to mark a token divides it
        for (int j = tid; j < n; j += kSampThreads) {
            const int t = a.seen[(size_t)b * a.max_seen + j];
            if (t < 0 || t >= V) continue;
            const unsigned m = 1u << (t & 31);
            if (!(atomicOr(&bits[t >> 5], m) & m)) p[t] = p[t] / a.penalty;
        }
        __syncthreads();
    }
    // 3. softmax
    float mx = -FLT_MAX;
    for (int i = tid; i < V; i += kSampThreads) mx = fmaxf(mx, p[i]);
    mx = block_reduce(mx, [](float x, float y) { return fmaxf(x, y); }, red_f);
    double sum = 0.0;
    for (int i = tid; i < V; i += kSampThreads) {
        const float e = expf(p[i] - mx);
        p[i] = e;
        sum += (double)e;
    }
    sum = block_reduce(sum, [](double x, double y) { return x + y; }, red_d);
    for (int i = tid; i < V; i += kSampThreads) p[i] = (float)((double)p[i] / sum);
    __syncthreads();

    const bool topk = a.top_k > 0 && a.top_k < V;
    const bool topp = a.top_p > 0.0f && a.top_p < 1.0f;
    if (topk) {
        // 4. the k-th largest (p, index) key by an 8-bit radix select, then
        //    everything below it set to 0
        const unsigned long long kth =
            block_radix_kth([&](int i) { return samp_key(p[i], i); }, V, a.top_k, hist, &s_keep, &s_count);
        for (int i = tid; i < V; i += kSampThreads)
            if (samp_key(p[i], i) < kth) p[i] = 0.0f;   // exactly top_k keys are >= kth
        __syncthreads();
    }
    if (topp) {
        // 5. the kept p > 0 sorted by (p, index) descending, their F32 running
        //    sum until it reaches top_p.  Taken kSampCand keys at a time: the
        //    round's keys are the largest below `hi` (a radix select finds the
        //    smallest of them when more remain), bitonic-sorted, and thread 0
        //    continues the running sum over them.
        unsigned long long hi = ~0ull;   // keys >= hi are in earlier rounds
        unsigned long long cut = 0ull;   // the nucleus: keys >= cut
        float cum = 0.0f;                // (thread 0)
        for (;;) {
            auto key_below = [&](int i) {
                const unsigned long long k = samp_key(p[i], i);
                return (p[i] > 0.0f && k < hi) ? k : 0ull;
            };
            int left = 0;
            for (int i = tid; i < V; i += kSampThreads) left += key_below(i) != 0ull;
            left = block_reduce(left, [](int x, int y) { return x + y; }, reinterpret_cast<int*>(red_f));
            if (left == 0) break;   // every kept key is in (the sum never reached top_p)
            const unsigned long long lo =
                left > kSampCand ? block_radix_kth(key_below, V, kSampCand, hist, &s_keep, &s_count) : 1ull;
            if (tid == 0) s_count = 0;
            __syncthreads();
            for (int i = tid; i < V; i += kSampThreads) {
                const unsigned long long k = key_below(i);
                if (k != 0ull && k >= lo) {
                    const int at = atomicAdd(&s_count, 1);
                    if (at < kSampCand) cand[at] = k;
                }
            }
            __syncthreads();
            const int n = min(s_count, kSampCand);
            for (int i = n + tid; i < kSampCand; i += kSampThreads) cand[i] = 0ull;
            __syncthreads();
            // bitonic sort, descending
            for (int size = 2; size <= kSampCand; size <<= 1) {
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    const int i = tid, j = i ^ stride;
                    if (j > i) {
                        const bool desc = (i & size) == 0;
                        const unsigned long long x = cand[i], y = cand[j];
                        if (desc ? (x < y) : (x > y)) {
                            cand[i] = y;
                            cand[j] = x;
                        }
                    }
                    __syncthreads();
                }
            }
            if (tid == 0) {
                int m = 0;
                bool reached = false;
                while (m < n) {
                    cum += __uint_as_float((unsigned)(cand[m] >> 32));
                    ++m;
                    if (cum >= a.top_p) {
                        reached = true;
                        break;
                    }
                }
                s_keep = reached ? 1 : 0;
                red_k[0] = cand[m - 1];   // the smallest key taken so far
            }
            __syncthreads();
            cut = red_k[0];
            const bool reached = s_keep != 0;
            __syncthreads();
            if (reached) break;
            hi = cut;
        }
        // zero every p outside the nucleus (its keys are the largest ones)
        if (cut != 0ull)
            for (int i = tid; i < V; i += kSampThreads)
                if (p[i] > 0.0f && samp_key(p[i], i) < cut) p[i] = 0.0f;
        __syncthreads();
    }
    // 6. renormalise
    double s2 = 0.0;
    for (int i = tid; i < V; i += kSampThreads) s2 += (double)p[i];
    s2 = block_reduce(s2, [](double x, double y) { return x + y; }, red_d);
    if (s2 <= 0.0) {
        // nothing left: the first index of the largest logit
        unsigned long long best = 0ull;
        for (int i = tid; i < V; i += kSampThreads) {
            const float v = lg[i];
            const unsigned ob = __float_as_uint(v);
            const unsigned ord = (ob & 0x80000000u) ? ~ob : (ob | 0x80000000u);
            const unsigned long long k = ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (unsigned)i);
            best = k > best ? k : best;
        }
        best = block_reduce(best, [](unsigned long long x, unsigned long long y) { return x > y ? x : y; }, red_k);
        if (tid == 0) a.out[b] = (int)(0xFFFFFFFFu - (unsigned)(best & 0xFFFFFFFFu));
        return;
    }
    for (int i = tid; i < V; i += kSampThreads) p[i] = (float)((double)p[i] / s2);
    __syncthreads();
    // 7. running F32 sum in index order, the reference's sequential loop.
    //    Zeros leave it unchanged, so each tile of kSampTile entries is
    //    compacted (block scan) to its nonzero entries in index order and
    //    thread 0 continues the sum over those from shared memory.
    const float u = a.u[b];
    if (u <= 0.0f) {   // index 0: its running sum is >= 0
        if (tid == 0) a.out[b] = 0;
        return;
    }
    const int lane = tid & 31, warp = tid >> 5;
    float acc = 0.0f;   // thread 0's running sum
    int tok = V - 1;
    if (tid == 0) s_token = -1;
    for (int base = 0; base < V; base += kSampTile) {
        float v[kSampPer];
        int c = 0;
#pragma unroll
        for (int j = 0; j < kSampPer; ++j) {
            const int i = base + tid * kSampPer + j;
            v[j] = i < V ? p[i] : 0.0f;
            c += v[j] != 0.0f;
        }
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) warp_cnt[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const int w = warp_cnt[lane];
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += t;
            }
            warp_cnt[lane] = wi - w;
            if (lane == 31) s_count = wi;
        }
        __syncthreads();
        int at = warp_cnt[warp] + incl - c;
#pragma unroll
        for (int j = 0; j < kSampPer; ++j)
            if (v[j] != 0.0f) {
                tile_v[at] = v[j];
                tile_i[at] = base + tid * kSampPer + j;
                ++at;
            }
        __syncthreads();
        if (tid == 0) {
            const int n = s_count;
            for (int m = 0; m < n; ++m) {
                acc += tile_v[m];
                if (u <= acc) {
                    s_token = tile_i[m];
                    break;
                }
            }
        }
        __syncthreads();
        if (s_token >= 0) {
            tok = s_token;
            break;
        }
    }
    if (tid == 0) a.out[b] = tok;
}

// ---------------------------------------------------------------------------
// The same steps with one thread-block cluster of kClu CTAs per row: each CTA
// keeps a slice of S probabilities in shared memory for every pass, and the
// row-wide values (max, sums, the radix histograms, the top-p candidates) are
// combined through distributed shared memory in rank order, so every CTA of
// the cluster derives the same thresholds.  Step 7's sequential sum hands its
// F32 running value from CTA to CTA in index order.  No work buffer; rows of
// up to kClu * kCluMaxSlice entries (the single-CTA kernel above takes longer
// rows).
// ---------------------------------------------------------------------------
constexpr int kClu = 8;
constexpr int kCluMaxSlice = 24576;

template <typename T, typename Op>
__device__ __forceinline__ T cluster_combine(cg::cluster_group& cl, T v, T* slot, T* all, Op op) {
    if (threadIdx.x == 0) *slot = v;
    cl.sync();
    if (threadIdx.x == 0) {
        T acc = *cl.map_shared_rank(slot, 0);
        for (int q = 1; q < kClu; ++q) acc = op(acc, *cl.map_shared_rank(slot, q));
        *all = acc;
    }
    cl.sync();   // also: every remote read of `slot` is done before it is written again
    return *all;
}

__global__ void __cluster_dims__(kClu, 1, 1) __launch_bounds__(kSampThreads)
sample_cluster_kernel(const __grid_constant__ SampArgs a, int S) {
    cg::cluster_group cl = cg::this_cluster();
    const int r = (int)cl.block_rank(), b = blockIdx.y, tid = threadIdx.x, V = a.vocab;
    const int lo = r * S;
    const int n = max(0, min(V, lo + S) - lo);   // this CTA's entries [lo, lo + n)
    extern __shared__ __align__(16) unsigned char samp_smem[];
    float* p = reinterpret_cast<float*>(samp_smem);   // [S]
    int* ix = reinterpret_cast<int*>(p + S);           // [S] step-7 compaction
    unsigned* bits = reinterpret_cast<unsigned*>(ix + S);   // [S / 32 + 1]
    __shared__ double red_d[32], x_d, all_d;
    __shared__ float red_f[32], x_f, all_f;
    __shared__ unsigned long long red_k[32], x_k, all_k;
    __shared__ unsigned long long loc[kSampCand], cand[kSampCand];
    __shared__ unsigned hist[2][256], comb[256];
    __shared__ int cnt_all[kClu], cnt_tile[32];
    __shared__ int s_loc, s_keep, s_need, s_nz, s_done;
    __shared__ float s_acc;
    const float* lg = a.logits + (size_t)b * a.ld + lo;

    // 1-2. temperature, then the repetition penalty on first occurrences (each
    //      CTA marks the seen tokens of its slice)
    const bool temp = a.temperature > 0.0f && a.temperature != 1.0f;
    for (int i = tid; i < n; i += kSampThreads) p[i] = temp ? lg[i] / a.temperature : lg[i];
    for (int i = tid; i < S / 32 + 1; i += kSampThreads) bits[i] = 0u;
    if (tid == 0) {
        s_acc = 0.0f;
        s_done = 0;
    }
    __syncthreads();
    if (a.penalty > 1.0f) {
        const int ns = min(a.n_seen[b], a.max_seen);
        for (int j = tid; j < ns; j += kSampThreads) {
            const int t = a.seen[(size_t)b * a.max_seen + j] - lo;
            if (t < 0 || t >= n) continue;
            const unsigned m = 1u << (t & 31);
            if (!(atomicOr(&bits[t >> 5], m) & m)) p[t] = p[t] / a.penalty;
        }
        __syncthreads();
    }
    // 3. softmax over the row
    float mx = -FLT_MAX;
    for (int i = tid; i < n; i += kSampThreads) mx = fmaxf(mx, p[i]);
    mx = block_reduce(mx, [](float x, float y) { return fmaxf(x, y); }, red_f);
    mx = cluster_combine(cl, mx, &x_f, &all_f, [](float x, float y) { return fmaxf(x, y); });
    double sum = 0.0;
    for (int i = tid; i < n; i += kSampThreads) {
        const float e = expf(p[i] - mx);
        p[i] = e;
        sum += (double)e;
    }
    sum = block_reduce(sum, [](double x, double y) { return x + y; }, red_d);
    sum = cluster_combine(cl, sum, &x_d, &all_d, [](double x, double y) { return x + y; });
    for (int i = tid; i < n; i += kSampThreads) p[i] = (float)((double)p[i] / sum);
    __syncthreads();

    const bool topk = a.top_k > 0 && a.top_k < V;
    const bool topp = a.top_p > 0.0f && a.top_p < 1.0f;
    if (topk) {
        // 4. radix select of the k-th largest key over the cluster's histograms
        unsigned long long prefix = 0ull, mask = 0ull;
        int need = a.top_k;
        int par = 0;
        for (int shift = 56; shift >= 0; shift -= 8, par ^= 1) {
            unsigned* h = hist[par];   // rewritten two passes later, after a cluster barrier
            for (int i = tid; i < 256; i += kSampThreads) h[i] = 0u;
            __syncthreads();
            for (int base = 0; base < n; base += kSampThreads) {
                const int i = base + tid;
                const unsigned long long k = i < n ? samp_key(p[i], lo + i) : 0ull;
                const bool hit = i < n && (k & mask) == prefix;
                const unsigned act = __ballot_sync(0xffffffffu, hit);
                if (hit) {
                    const unsigned bin = (unsigned)(k >> shift) & 255u;
                    const unsigned peers = __match_any_sync(act, bin);
                    if ((tid & 31) == __ffs(peers) - 1) atomicAdd(&h[bin], (unsigned)__popc(peers));
                }
            }
            cl.sync();
            if (tid < 256) {
                unsigned c = 0u;
                for (int q = 0; q < kClu; ++q) c += cl.map_shared_rank(h, q)[tid];
                comb[tid] = c;
            }
            __syncthreads();
            if (tid < 32) radix_pick(comb, need, &s_keep, &s_need);
            __syncthreads();
            prefix |= (unsigned long long)s_keep << shift;
            mask |= 255ull << shift;
            need = s_need;
            __syncthreads();
        }
        for (int i = tid; i < n; i += kSampThreads)
            if (samp_key(p[i], lo + i) < prefix) p[i] = 0.0f;
        __syncthreads();
    }
    if (topp) {
        // 5. every CTA gathers the cluster's kept p > 0 (at most top_k <= 1024)
        //    in rank order and sorts them
        if (tid == 0) s_loc = 0;
        __syncthreads();
        for (int i = tid; i < n; i += kSampThreads)
            if (p[i] > 0.0f) {
                const int at = atomicAdd(&s_loc, 1);
                if (at < kSampCand) loc[at] = samp_key(p[i], lo + i);
            }
        cl.sync();
        if (tid < kClu) cnt_all[tid] = min(*cl.map_shared_rank(&s_loc, tid), kSampCand);
        __syncthreads();
        int total = 0;
        for (int q = 0; q < kClu; ++q) {
            const unsigned long long* rl = cl.map_shared_rank(loc, q);
            for (int i = tid; i < cnt_all[q] && total + i < kSampCand; i += kSampThreads) cand[total + i] = rl[i];
            total += cnt_all[q];
        }
        total = min(total, kSampCand);
        for (int i = total + tid; i < kSampCand; i += kSampThreads) cand[i] = 0ull;
        cl.sync();   // the remote reads of loc / s_loc are done
        int P = 2;   // the sort covers the first P >= total entries (the rest are zero)
        while (P < total) P <<= 1;
        for (int size = 2; size <= P; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                const int i = tid, j = i ^ stride;
                if (i < P && j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long x = cand[i], y = cand[j];
                    if (desc ? (x < y) : (x > y)) {
                        cand[i] = y;
                        cand[j] = x;
                    }
                }
                __syncthreads();
            }
        }
        if (tid == 0) {
            float cum = 0.0f;
            int m = 0;
            while (m < total) {
                cum += __uint_as_float((unsigned)(cand[m] >> 32));
                ++m;
                if (cum >= a.top_p) break;
            }
            s_keep = m;
        }
        __syncthreads();
        const int m = s_keep;
        const unsigned long long kmin = m > 0 ? cand[m - 1] : ~0ull;
        for (int i = tid; i < n; i += kSampThreads)
            if (p[i] > 0.0f && samp_key(p[i], lo + i) < kmin) p[i] = 0.0f;
        __syncthreads();
    }
    // 6. renormalise
    double s2 = 0.0;
    for (int i = tid; i < n; i += kSampThreads) s2 += (double)p[i];
    s2 = block_reduce(s2, [](double x, double y) { return x + y; }, red_d);
    s2 = cluster_combine(cl, s2, &x_d, &all_d, [](double x, double y) { return x + y; });
    if (s2 <= 0.0) {
        unsigned long long best = 0ull;
        for (int i = tid; i < n; i += kSampThreads) {
            const unsigned ob = __float_as_uint(lg[i]);
            const unsigned ord = (ob & 0x80000000u) ? ~ob : (ob | 0x80000000u);
            const unsigned long long k = ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (unsigned)(lo + i));
            best = k > best ? k : best;
        }
        auto kmax = [](unsigned long long x, unsigned long long y) { return x > y ? x : y; };
        best = block_reduce(best, kmax, red_k);
        best = cluster_combine(cl, best, &x_k, &all_k, kmax);
        if (r == 0 && tid == 0) a.out[b] = (int)(0xFFFFFFFFu - (unsigned)(best & 0xFFFFFFFFu));
        return;
    }
    const float u = a.u[b];
    if (u <= 0.0f) {   // index 0: its running sum is >= 0
        if (r == 0 && tid == 0) a.out[b] = 0;
        return;
    }
    // 7. this slice's nonzero p / s2 compacted in index order (in place: a tile
    //    is read into registers before any of it is overwritten)
    const int lane = tid & 31, warp = tid >> 5;
    int off = 0;
    for (int base = 0; base < n; base += kSampTile) {
        float v[kSampPer];
        int c = 0;
#pragma unroll
        for (int j = 0; j < kSampPer; ++j) {
            const int i = base + tid * kSampPer + j;
            v[j] = i < n ? (float)((double)p[i] / s2) : 0.0f;
            c += v[j] != 0.0f;
        }
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) cnt_tile[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const int w = cnt_tile[lane];
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += t;
            }
            cnt_tile[lane] = wi - w;
            if (lane == 31) s_nz = wi;
        }
        __syncthreads();
        int at = off + cnt_tile[warp] + incl - c;
#pragma unroll
        for (int j = 0; j < kSampPer; ++j)
            if (v[j] != 0.0f) {
                p[at] = v[j];
                ix[at] = lo + base + tid * kSampPer + j;
                ++at;
            }
        off += s_nz;
        __syncthreads();
    }
    //    the F32 running sum, CTA by CTA in rank (= index) order
    for (int q = 0; q < kClu; ++q) {
        if (r == q && tid == 0) {
            float acc = s_acc;
            int done = s_done;
            for (int m = 0; m < off && !done; ++m) {
                acc += p[m];
                if (u <= acc) {
                    a.out[b] = ix[m];
                    done = 1;
                }
            }
            if (q + 1 < kClu) {
                *cl.map_shared_rank(&s_acc, q + 1) = acc;
                *cl.map_shared_rank(&s_done, q + 1) = done;
            } else if (!done) {
                a.out[b] = V - 1;
            }
        }
        cl.sync();
    }
}

// ---------------------------------------------------------------------------
// Log-probabilities of scored tokens (Model::score_logprobs, model.cpp:1746-
// 1831): per row of logits [n][V], lp = (l - max) - log(sum exp(l - max)),
// the target token's lp and the k largest lps (descending; equal lps: the
// smaller index first).  One CTA of 1024 threads per row; the top k by the
// 8-bit radix select of the sampler on order-preserving keys.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long lp_key(float v, int i) {
    const unsigned b = __float_as_uint(v);
    const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);   // float order as unsigned order
    return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (unsigned)i);   // equal values: smaller index larger
}

__global__ void __launch_bounds__(kSampThreads)
logprob_kernel(const float* __restrict__ logits, int V, int ld, const int* __restrict__ target, int k,
               float* __restrict__ out_lp, int* __restrict__ out_ids, float* __restrict__ out_top) {
    const int r = blockIdx.x, tid = threadIdx.x;
    const float* lg = logits + (size_t)r * ld;
    __shared__ float red_f[32];
    __shared__ unsigned long long cand[kSampCand];
    __shared__ int s_keep, s_count;
    __shared__ unsigned hist[256];
    float mx = -1e30f;   // model.cpp:1793
    for (int i = tid; i < V; i += kSampThreads) mx = fmaxf(mx, lg[i]);
    mx = block_reduce(mx, [](float x, float y) { return fmaxf(x, y); }, red_f);
    float se = 0.f;
    for (int i = tid; i < V; i += kSampThreads) se += expf(lg[i] - mx);
    se = block_reduce(se, [](float x, float y) { return x + y; }, red_f);
    const float lse = logf(se);
    auto lp = [&](int i) { return (lg[i] - mx) - lse; };
    if (tid == 0) out_lp[r] = lp(target[r]);
    if (k <= 0) return;
    // the k-th largest key
    unsigned long long prefix = 0ull, mask = 0ull;
    int need = k;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kSampThreads) hist[i] = 0u;
        __syncthreads();
        for (int i = tid; i < V; i += kSampThreads) {
            const unsigned long long key = lp_key(lp(i), i);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid < 32) radix_pick(hist, need, &s_keep, &s_count);
        __syncthreads();
        prefix |= (unsigned long long)s_keep << shift;
        mask |= 255ull << shift;
        need = s_count;
        __syncthreads();
    }
    if (tid == 0) s_count = 0;
    __syncthreads();
    for (int i = tid; i < V; i += kSampThreads) {
        const unsigned long long key = lp_key(lp(i), i);
        if (key >= prefix) {
            const int at = atomicAdd(&s_count, 1);
            if (at < kSampCand) cand[at] = key;
        }
    }
    __syncthreads();
    for (int i = min(s_count, kSampCand) + tid; i < kSampCand; i += kSampThreads) cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= kSampCand; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const int i = tid, j = i ^ stride;
            if (j > i) {
                const bool desc = (i & size) == 0;
                const unsigned long long x = cand[i], y = cand[j];
                if (desc ? (x < y) : (x > y)) {
                    cand[i] = y;
                    cand[j] = x;
                }
            }
            __syncthreads();
        }
    }
    if (tid < k) {
        const int id = (int)(0xFFFFFFFFu - (unsigned)(cand[tid] & 0xFFFFFFFFu));
        out_ids[(size_t)r * k + tid] = id;
        out_top[(size_t)r * k + tid] = lp(id);
    }
}

tvb_status logprob_rows(const float* logits, int n, int V, int ld, const int* target, int k, float* out_lp,
                        int* out_ids, float* out_top, cudaStream_t st) {
    TVB_REQUIRE(logits && target && out_lp && n > 0 && V > 0 && k >= 0 && k <= kMaxLogprobs && (k == 0 || (out_ids && out_top)),
                "logprobs: bad arguments (k %d, at most %d)", k, kMaxLogprobs);
    logprob_kernel<<<n, kSampThreads, 0, st>>>(logits, V, ld, target, k, out_lp, out_ids, out_top);
    return check_launch("logprob_kernel");
}

}  // namespace tvb

extern "C" tvb_status tvb_sample(const float* logits, int B, int vocab, int ld, const tvb_sampler_config* cfg,
                                 const int* seen, const int* n_seen, int max_seen, const float* u, int* out,
                                 void* stream) {
    using namespace tvb;
    TVB_REQUIRE(logits && cfg && u && out && B > 0 && vocab > 0 && ld >= vocab, "sample: bad arguments");
    TVB_REQUIRE(!(cfg->repetition_penalty > 1.0f) || (seen && n_seen && max_seen >= 0),
                "sample: repetition penalty needs the seen tokens");
    const bool topp = cfg->top_p > 0.0f && cfg->top_p < 1.0f;
    // top-p over more than kSampCand candidates (top_k 0 = the whole vocabulary,
    // or top_k above kSampCand): the one-CTA kernel, whose nucleus search takes
    // kSampCand keys a round
    const bool wide_nucleus = topp && !(cfg->top_k >= 1 && cfg->top_k <= kSampCand);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    SampArgs a;
    a.logits = logits;
    a.vocab = vocab;
    a.ld = ld;
    a.temperature = cfg->temperature;
    a.penalty = cfg->repetition_penalty;
    a.top_p = cfg->top_p;
    a.top_k = cfg->top_k;
    a.seen = seen;
    a.n_seen = n_seen;
    a.max_seen = max_seen;
    a.u = u;
    a.out = out;
    a.work = nullptr;
    a.bits = nullptr;
    const int S = ((vocab + kClu - 1) / kClu + 31) / 32 * 32;   // entries per CTA of a row's cluster
    if (S <= kCluMaxSlice && !wide_nucleus) {
        const size_t smem = (size_t)S * 8 + ((size_t)S / 32 + 1) * 4;
        static size_t smem_set = 0;
        if (smem > smem_set) {
            TVB_CUDA(cudaFuncSetAttribute(sample_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
            smem_set = smem;
        }
        sample_cluster_kernel<<<dim3(kClu, (unsigned)B), kSampThreads, smem, st>>>(a, S);
        return check_launch("sample_cluster_kernel");
    }
    const size_t words = (size_t)vocab / 32 + 1;
    void* ws = nullptr;
    TVB_CUDA(cudaMallocAsync(&ws, (size_t)B * ((size_t)vocab * 4 + words * 4), st));
    a.work = static_cast<float*>(ws);
    a.bits = reinterpret_cast<unsigned*>(static_cast<float*>(ws) + (size_t)B * vocab);
    sample_kernel<<<B, kSampThreads, 0, st>>>(a);
    const cudaError_t le = cudaGetLastError();
    cudaFreeAsync(ws, st);
    if (le != cudaSuccess) return cuda_error(le, "sample_kernel");
    return TVB_OK;
}
