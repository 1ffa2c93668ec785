// Context (the state CUDABackend::Impl owns, cuda/ops_cuda.cu:309-591) and the
// fused, graph-captured decode step replacing Model::forward_gpu
// (src/model.cpp:1354-1582).
//
// One decode step = per layer [QKV+RoPE+KV append] -> [attention] ->
// [sub-norm + o_proj + residual] -> [ffn_norm + gate/up + relu^2*up] ->
// [sub-norm + down + residual], then [output_norm + lm_head + argmax]:
// 5 kernels per layer + 1, launched with programmatic dependent launch and
// captured once into a CUDA graph.  Position and token live in device memory
// (StepState), so the same graph serves every position and greedy decode can
// chain steps without the host.
#include "decode.cuh"
#include "prefill.h"
#include "tp_prefill.h"
#include "batch_decode.h"
#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>


namespace tvb {

__device__ unsigned g_standalone_status;

// TVB_DISABLE_PDL=1 launches the fused step without programmatic dependent
// launch (for profilers and A/B timing); read once when a context is created.
static bool g_disable_pdl = false;

template <typename... KArgs, typename... Args>
static cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && !g_disable_pdl) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Largest dynamic shared memory a GEMV launch may request: the device's
// opt-in per-block limit minus a margin for the kernels' static shared memory.
static int g_max_dyn_smem = 0;

template <int MODE, int WT, int R, bool TP = false>
static tvb_status launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
    const int units = gemv_units<MODE>(a, R);
    if (units <= 0) return TVB_OK;
    const int grid = std::min(units, num_sms());
    const GemvSmem L = gemv_smem_layout(a.K, WT == WT_F16 ? 2 : 1, gemv_rows_cap(units, grid, R));
    if (L.total > g_max_dyn_smem)
        return set_error(TVB_ERR_UNSUPPORTED, "gemv: K=%d too large for shared-memory staging", a.K);
    auto kern = stream_gemv_kernel<MODE, WT, R, TP>;
    TVB_CUDA(launch_ex(kern, dim3(grid), dim3(kGemvThreads), (size_t)L.total, st, pdl, a));
    return TVB_OK;
}

// Opt every GEMV instantiation into the full dynamic shared memory once, before
// any launch (and outside stream capture).
template <int MODE, int WT, int R>
static cudaError_t allow_smem() {
    return cudaFuncSetAttribute(stream_gemv_kernel<MODE, WT, R>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, g_max_dyn_smem);
}

tvb_status prepare_kernels() {
    static int done = 0;
    if (done) return TVB_OK;
    int dev = 0, optin = 0;
    TVB_CUDA(cudaGetDevice(&dev));
    TVB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    g_max_dyn_smem = optin - 1024;
    cudaError_t e = cudaSuccess;
    cudaError_t r[] = {
        allow_smem<GM_PLAIN, WT_F16, 1>(), allow_smem<GM_PLAIN, WT_I8, 1>(),
        allow_smem<GM_QKV, WT_F16, 2>(),   allow_smem<GM_QKV, WT_I8, 2>(),
        allow_smem<GM_RESID, WT_F16, 1>(), allow_smem<GM_RESID, WT_I8, 1>(),
        allow_smem<GM_GATEUP, WT_F16, 2>(), allow_smem<GM_GATEUP, WT_I8, 2>(),
        allow_smem<GM_LMHEAD, WT_F16, 1>(),
        cudaFuncSetAttribute(stream_gemv_kernel<GM_LMHEAD, WT_F16, 1, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, g_max_dyn_smem),
    };
    for (cudaError_t x : r)
        if (x != cudaSuccess) e = x;
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute");
    num_sms();
    done = 1;
    return TVB_OK;
}

// Weight-type dispatch for the fused modes.
template <int MODE, int R>
static tvb_status launch_gemv_wt(int wt, const GemvArgs& a, cudaStream_t st, bool pdl) {
    return wt == WT_F16 ? launch_gemv<MODE, WT_F16, R>(a, st, pdl)
                        : launch_gemv<MODE, WT_I8, R>(a, st, pdl);
}

static tvb_status launch_attn(const AttnArgs& a, cudaStream_t st, bool pdl) {
    TVB_CUDA(launch_ex(attn_decode_kernel, dim3(a.nkv, a.nsplit), dim3(kAttnThreads), 0, st, pdl, a));
    return TVB_OK;
}

static bool wt_of(tvb_dtype d, int* wt) {
    if (d == TVB_F16) { *wt = WT_F16; return true; }
    if (d == TVB_I8_ROW || d == TVB_I8_TENSOR) { *wt = WT_I8; return true; }
    return false;
}

static void fill_weight(GemvArgs& a, int slot, const tvb_weight& w) {
    a.w[slot] = w.w;
    a.row_scale[slot] = (w.dtype == TVB_I8_ROW) ? w.row_scales : nullptr;
    a.tscale[slot] = (w.dtype == TVB_I8_TENSOR) ? w.tensor_scale : 1.0f;
}

}  // namespace tvb

using namespace tvb;

struct tvb_context {
    tvb_model_config cfg;
    int H, Hq, Hk, I, V, L;
    int device;
    cudaStream_t stream = nullptr;
    // reference-API activation buffers (ops.h:94-110)
    float *d_x = nullptr, *d_norm = nullptr, *d_q = nullptr, *d_k = nullptr, *d_v = nullptr,
          *d_gate = nullptr, *d_up = nullptr;
    float *h_qkv = nullptr, *h_attn = nullptr, *h_logit = nullptr;
    // fused-step buffers
    float *e_x = nullptr, *e_q = nullptr, *e_attn = nullptr, *e_h = nullptr, *e_logits = nullptr;
    float* attn_part = nullptr;
    int nsplit = 8;    // attention splits per KV head, merged by the o_proj phase
    float *kcache = nullptr, *vcache = nullptr;   // slots x [L][max_seq][Hk]; slot 0 is the step's
    int slots = 1;                                // KV cache slots (batched decode)
    size_t slot_floats = 0;                       // floats per slot
    float *rope_cos = nullptr, *rope_sin = nullptr;
    StepState* st = nullptr;
    int* hist = nullptr;
    // pinned staging
    StepState* h_st = nullptr;
    int* h_io = nullptr;       // [max_seq][2] (pos, token) staging for prefill steps
    int* h_hist = nullptr;
    // weights
    std::vector<tvb_layer_weights> layers;
    std::vector<bool> layer_set;
    const void* tok_embd = nullptr;
    const float* output_norm = nullptr;
    // the decode step as a phase table for decode_step_kernel
    Phase* d_phases = nullptr;
    int n_phases = 0;
    int step_smem = 0;
    // graphs
    cudaGraphExec_t g_step = nullptr;    // layers + lm_head
    cudaGraphExec_t g_layers = nullptr;  // layers only (prefill rows before the last)
    bool dirty = true;
    unsigned gen = 0;   // weights / tensor-parallel setup changes (invalidate captured graphs)
    // the batched step as a graph per batch size: a size is run once eagerly
    // (lazy set-up: kernel attributes, scratch) and captured on its next call
    cudaGraphExec_t bd_graph = nullptr;
    int bd_graph_B = 0;
    unsigned bd_gen = 0;
    unsigned long long bd_eager = 0;   // bit B: run eagerly at generation bd_gen
    // batched-prefill workspace (allocated by the first tvb_prefill): rows of
    // the prompt chunk in flight, F16 hi/lo activation planes for the tensor
    // cores, and the F16 widening of one projection group of an INT8 layer
    int pf_cap = 0;
    float *pf_x = nullptr, *pf_q = nullptr, *pf_attn = nullptr, *pf_h = nullptr;
    uint16_t *pf_xh = nullptr, *pf_xl = nullptr;
    int *pf_exp = nullptr, *pf_tok = nullptr;
    void* pf_planes = nullptr;   // F16 hi/lo q, K, V^T planes of the tensor-core attention
    // tensor parallelism (tvb_tp_init / tvb_tp_set_peers): this rank's exchange
    // buffer, every rank's (IPC-mapped) buffer, and a second residual vector
    // (folds alternate between e_x and e_x2)
    int tp_world = 1, tp_rank = 0;
    float* tp_xchg = nullptr;
    float* tp_peer[kMaxTp] = {};
    bool tp_ready = false;
    // a device-side wait of a tensor-parallel step gave up: the exchange
    // counters of the ranks no longer agree, so steps are refused until every
    // rank has called tvb_tp_recover
    bool tp_failed = false;
    float* e_x2 = nullptr;
    int n_push = 0;   // row-parallel exchanges per launch (both graphs)
    size_t tp_xf_off = 0;   // float offset of the decode step's row-exchange flags
    size_t tp_pf_off = 0;   // float offset of the prefill region in every rank's exchange buffer
    size_t tp_key_off = 0;  // float offset of the batched step's argmax keys
    // batched decode / split-K workspace (pf_workspace)
    float* pf_part = nullptr;   // split-K partial sums / stream-K pieces
    unsigned* pf_flags = nullptr;   // stream-K piece flags [SMs][4]
    size_t pf_part_floats = 0;
    float* bd_attn_part = nullptr;   // [max_batch][nh][splits][hd + 4]
    float* bd_logits = nullptr;      // [max_batch][V]
    int* bd_io = nullptr;            // [tokens | positions | next tokens] x kMaxBatch
    unsigned long long* bd_keys = nullptr;
    float* pf_inv = nullptr;   // per-row 1/rms of a tensor-parallel sub-norm
    uint16_t* pf_w16 = nullptr;
    size_t pf_w16_elems = 0;
};

namespace {

tvb_status alloc_dev(void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc");
    return TVB_OK;
}

// The decode step as phases (src/model.cpp:1399-1451, 1571-1580).
std::vector<Phase> build_phases(tvb_context* c) {
    std::vector<Phase> ph;
    const float scale = 1.0f / std::sqrt((float)c->cfg.head_dim);
    // Tensor parallelism: q/k/v and gate/up are this rank's rows, o_proj and
    // down its columns; those two end with an exchange of partial rows and the
    // phase after each folds them into the residual (alternating buffers).
    const bool tp = c->tp_world > 1;
    TpArgs tpb = {};
    if (tp) {
        tpb.world = c->tp_world;
        tpb.rank = c->tp_rank;
        tpb.ld = c->H + 4;
        tpb.xf_off = (int)c->tp_xf_off;
        for (int r = 0; r < c->tp_world; ++r) tpb.peer[r] = c->tp_peer[r];
        tpb.index = -1;
        tpb.fold = -1;
    }
    float* xres[2] = {c->e_x, c->e_x2};
    int cur = 0;            // residual buffer the next phase reads
    int xi = 0;             // exchanges so far
    int fold_norm = 0;      // full length of the sub-norm of the last exchange (0: none)
    auto fold_into = [&](Phase& p) {
        p.g.x = xres[cur];
        if (tp && xi > 0) {
            p.g.tp.fold = xi - 1;
            p.g.tp.norm_n = fold_norm;
            p.g.tp.x_out = xres[cur ^ 1];
            p.g.x = xres[cur];
            cur ^= 1;
        }
    };
    auto gemv = [&](int mode, int wt) {
        Phase p = {};
        p.kind = PK_GEMV;
        p.mode = mode;
        p.wt = wt;
        p.g.eps = c->cfg.rms_norm_eps;
        p.g.st = c->st;
        p.g.status = &c->st->status;
        p.g.tp = tpb;
        return p;
    };
    for (int l = 0; l < c->L; ++l) {
        const tvb_layer_weights& lw = c->layers[l];
        int wt = WT_F16;
        wt_of(lw.wq.dtype, &wt);
        float* kl = c->kcache + (size_t)l * c->cfg.max_seq_len * c->Hk;
        float* vl = c->vcache + (size_t)l * c->cfg.max_seq_len * c->Hk;
        {   // (a)-(c): attn_norm, q/k/v, RoPE, KV append
            Phase p = gemv(GM_QKV, wt);
            fill_weight(p.g, 0, lw.wq);
            fill_weight(p.g, 1, lw.wk);
            fill_weight(p.g, 2, lw.wv);
            p.g.K = c->H;
            if (l == 0) cur = 0;
            else fold_into(p);
            if (l == 0) p.g.x = xres[0];
            p.g.embd = static_cast<const uint16_t*>(c->tok_embd);
            p.g.x_out = xres[0];
            p.g.gather_token = (l == 0);
            p.g.norm_w = lw.attn_norm;
            p.g.nh = c->cfg.num_heads;
            p.g.nkv = c->cfg.num_kv_heads;
            p.g.hd = c->cfg.head_dim;
            p.g.q_out = c->e_q;
            p.g.kcache = kl;
            p.g.vcache = vl;
            p.g.rope_cos = c->rope_cos;
            p.g.rope_sin = c->rope_sin;
            ph.push_back(p);
        }
        {   // (d): attention over kv_len = pos + 1
            Phase p = {};
            p.kind = PK_ATTN;
            p.at.q = c->e_q;
            p.at.kcache = kl;
            p.at.vcache = vl;
            p.at.out = c->e_attn;
            p.at.part = c->attn_part;
            p.at.nh = c->cfg.num_heads;
            p.at.nkv = c->cfg.num_kv_heads;
            p.at.hd = c->cfg.head_dim;
            p.at.nsplit = c->nsplit;
            p.at.scale = scale;
            p.at.kv_len = -1;
            p.at.st = c->st;
            p.at.status = &c->st->status;
            ph.push_back(p);
        }
        {   // (e)-(f): attn_sub_norm, wo, residual
            Phase p = gemv(GM_RESID, wt);
            fill_weight(p.g, 0, lw.wo);
            p.g.N = c->H;
            p.g.K = c->Hq;
            p.g.x = c->e_attn;
            p.g.attn_part = c->attn_part;   // input: merge of the attention splits
            p.g.attn_nsplit = c->nsplit;
            p.g.hd = c->cfg.head_dim;
            p.g.norm_w = lw.attn_sub_norm;
            p.g.y = xres[cur];
            if (tp) {
                p.g.tp.index = xi++;
                fold_norm = lw.attn_sub_norm ? c->Hq * c->tp_world : 0;
            }
            ph.push_back(p);
        }
        {   // (g)-(h): ffn_norm, gate/up, relu^2 * up
            Phase p = gemv(GM_GATEUP, wt);
            fill_weight(p.g, 0, lw.w_gate);
            fill_weight(p.g, 1, lw.w_up);
            p.g.N = c->I;
            p.g.K = c->H;
            fold_into(p);
            p.g.norm_w = lw.ffn_norm;
            p.g.y = c->e_h;
            ph.push_back(p);
        }
        {   // (i): ffn_sub_norm, down, residual
            Phase p = gemv(GM_RESID, wt);
            fill_weight(p.g, 0, lw.w_down);
            p.g.N = c->H;
            p.g.K = c->I;
            p.g.x = c->e_h;
            p.g.norm_w = lw.ffn_sub_norm;
            p.g.y = xres[cur];
            if (tp) {
                p.g.tp.index = xi++;
                fold_norm = lw.ffn_sub_norm ? c->I * c->tp_world : 0;
            }
            ph.push_back(p);
        }
    }
    c->n_push = xi;
    {   // final norm + tied lm_head + argmax
        Phase p = gemv(GM_LMHEAD, WT_F16);
        const int vs = c->V / c->tp_world;   // this rank's vocabulary slice
        p.g.w[0] = static_cast<const uint16_t*>(c->tok_embd) + (size_t)c->tp_rank * vs * c->H;
        p.g.tscale[0] = 1.0f;
        p.g.N = vs;
        p.g.K = c->H;
        fold_into(p);
        p.g.norm_w = c->output_norm;
        p.g.y = c->e_logits;
        if (tp) {
            p.g.tp.vocab0 = c->tp_rank * vs;
            p.g.tp.index = 0;   // the launch's argmax exchange over the ranks' slices
        }
        ph.push_back(p);
    }
    return ph;
}

int phase_units(const Phase& p) {
    const int R = (p.mode == GM_QKV || p.mode == GM_GATEUP) ? 2 : 1;
    if (p.mode == GM_QKV) return (p.g.nh + 2 * p.g.nkv) * (p.g.hd >> 1);
    if (p.mode == GM_GATEUP) return p.g.N;
    return (p.g.N + R - 1) / R;
}

tvb_status capture(tvb_context* c, int n_phases, int n_argmax, cudaGraphExec_t* out) {
    if (*out) {
        cudaGraphExecDestroy(*out);
        *out = nullptr;
    }
    TVB_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = (size_t)c->step_smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t le = c->tp_world > 1
                         ? cudaLaunchKernelEx(&cfg, decode_step_kernel<true>, (const Phase*)c->d_phases,
                                              n_phases, c->st, c->n_push, n_argmax)
                         : cudaLaunchKernelEx(&cfg, decode_step_kernel<false>, (const Phase*)c->d_phases,
                                              n_phases, c->st, 0, 0);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (le != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return cuda_error(le, "launch decode_step_kernel");
    }
    if (e != cudaSuccess) return cuda_error(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_error(e, "cudaGraphInstantiate");
    return TVB_OK;
}

tvb_status ensure_graphs(tvb_context* c) {
    if (!c->dirty) return TVB_OK;
    for (int l = 0; l < c->L; ++l)
        if (!c->layer_set[l]) return set_error(TVB_ERR_STATE, "layer %d weights not set", l);
    if (!c->tok_embd || !c->output_norm) return set_error(TVB_ERR_STATE, "output weights not set");
    if (c->tp_world > 1 && !c->tp_ready)
        return set_error(TVB_ERR_STATE, "tensor parallelism: peers not set (tvb_tp_set_peers)");
    std::vector<Phase> ph = build_phases(c);
    // shared memory: the largest per-phase layout, and the attention scratch
    const int G = num_sms();
    int smem = 1024 + attn_item_smem(c->cfg.num_heads / c->cfg.num_kv_heads, c->cfg.head_dim);
    for (const Phase& p : ph) {
        if (p.kind != PK_GEMV) continue;
        const int R = (p.mode == GM_QKV || p.mode == GM_GATEUP) ? 2 : 1;
        const int units = phase_units(p);
        const GemvSmem L = gemv_smem_layout(p.g.K, p.wt == WT_F16 ? 2 : 1, gemv_rows_cap(units, G, R));
        smem = std::max(smem, L.total);
    }
    if (smem > g_max_dyn_smem)
        return set_error(TVB_ERR_UNSUPPORTED, "decode step needs %d B of shared memory", smem);
    auto kern = c->tp_world > 1 ? decode_step_kernel<true> : decode_step_kernel<false>;
    TVB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int per_sm = 0;
    TVB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, smem));
    if (per_sm < 1) return set_error(TVB_ERR_UNSUPPORTED, "decode step kernel cannot be resident");
    if (c->d_phases) cudaFree(c->d_phases);
    c->d_phases = nullptr;
    TVB_TRY(alloc_dev((void**)&c->d_phases, ph.size() * sizeof(Phase)));
    TVB_CUDA(cudaMemcpy(c->d_phases, ph.data(), ph.size() * sizeof(Phase), cudaMemcpyHostToDevice));
    c->n_phases = (int)ph.size();
    c->step_smem = smem;
    TVB_TRY(capture(c, c->n_phases, 1, &c->g_step));
    TVB_TRY(capture(c, c->n_phases - 1, 0, &c->g_layers));
    c->dirty = false;
    return TVB_OK;
}

tvb_status check_status(tvb_context* c) {
    const unsigned s = c->h_st->status;
    if (!s) return TVB_OK;
    // clear counters, flags and the abort latch so the next call starts clean
    cudaMemsetAsync(c->st, 0, sizeof(StepState), c->stream);
    cudaStreamSynchronize(c->stream);
    // Under tensor parallelism the ranks' exchange buffers still hold arrival
    // counts and flags of the abandoned step, which the restarted counters
    // would compare against: no step may run until every rank recovers.
    if (c->tp_world > 1) c->tp_failed = true;
    if (s & kStatusTimeout) return set_error(TVB_ERR_TIMEOUT, "a device-side wait exceeded its limit");
    return set_error(TVB_ERR_CUDA, "device status 0x%x", s);
}

// Entry guard of every call that runs a (possibly tensor-parallel) step.
tvb_status tp_guard(const tvb_context* c, const char* what) {
    if (c->tp_world > 1 && c->tp_failed)
        return set_error(TVB_ERR_STATE,
                         "%s: a tensor-parallel step failed on this rank; call tvb_tp_recover on every rank first", what);
    return TVB_OK;
}

// ---- batched prefill (Model::forward_prefill, model.cpp:1139-1234) -----------------

// Split-K partial sums of the tensor-core GEMM: a split is chosen only while
// (tiles x row blocks x splits) fits the SMs, so rows-per-row-block x SMs x 256
// columns bounds every projection's partials.
constexpr int kPfPartRows = 128;

tvb_status pf_workspace(tvb_context* c) {
    if (c->pf_cap) return TVB_OK;
    const int cap = std::min(c->cfg.max_prefill, c->cfg.max_seq_len);
    const size_t kmax = (size_t)std::max(c->H, std::max(c->Hq, c->I));
    struct { void** p; size_t b; } allocs[] = {
        {(void**)&c->pf_x, (size_t)cap * c->H * 4},   {(void**)&c->pf_q, (size_t)cap * c->Hq * 4},
        {(void**)&c->pf_attn, (size_t)cap * c->Hq * 4}, {(void**)&c->pf_h, (size_t)cap * c->I * 4},
        {(void**)&c->pf_xh, cap * kmax * 2},          {(void**)&c->pf_xl, cap * kmax * 2},
        {(void**)&c->pf_exp, (size_t)cap * 4},        {(void**)&c->pf_tok, (size_t)c->cfg.max_seq_len * 4},
        {(void**)&c->pf_inv, (size_t)cap * 4},
        {(void**)&c->pf_part, (size_t)kPfPartRows * num_sms() * 256 * 4},
        {(void**)&c->bd_attn_part, (size_t)c->slots * c->cfg.num_heads * kMaxAttnSplits * (c->cfg.head_dim + 4) * 4},
        {(void**)&c->bd_logits, (size_t)c->slots * c->V * 4},
        {(void**)&c->bd_io, (size_t)3 * kMaxBatch * 4},
        {(void**)&c->bd_keys, (size_t)kMaxBatch * 8},
    };
    for (auto& a : allocs) TVB_TRY(alloc_dev(a.p, a.b));
    TVB_TRY(alloc_dev((void**)&c->pf_flags, (size_t)num_sms() * 4 * sizeof(unsigned)));
    TVB_CUDA(cudaMemset(c->pf_flags, 0, (size_t)num_sms() * 4 * sizeof(unsigned)));
    c->pf_part_floats = (size_t)kPfPartRows * num_sms() * 256;
    if (pf_attention_tc_supported(c->cfg.num_heads, c->cfg.num_kv_heads, c->cfg.head_dim))
        TVB_TRY(alloc_dev(&c->pf_planes, pf_attn_planes_bytes(cap, c->cfg.max_seq_len, c->cfg.num_heads,
                                                              c->cfg.num_kv_heads)));
    c->pf_cap = cap;
    return TVB_OK;
}

// The batched prefill tiles K by 64 (every projection's input width), gate/up
// rows by 32 and the attention's 64-row blocks by whole query-head groups.
bool pf_batched_supported(const tvb_context* c) {
    const int group = c->cfg.num_heads / c->cfg.num_kv_heads;
    return c->H % 64 == 0 && c->Hq % 64 == 0 && c->I % 64 == 0 && 64 % group == 0;
}

// One projection operand; INT8 weights are widened to F16 into the scratch at
// `off` (exact), their scales applied by the GEMM epilogue.
tvb_status pf_operand(tvb_context* c, const tvb_weight& w, int rows, int K, size_t& off, PfMatrix& m,
                      bool pdl = false) {
    m.rows = rows;
    m.row_scales = nullptr;
    m.scale = 1.0f;
    m.widened = w.dtype != TVB_F16;
    if (w.dtype == TVB_F16) {
        m.w = static_cast<const uint16_t*>(w.w);
        return TVB_OK;
    }
    TVB_REQUIRE(w.dtype == TVB_I8_ROW || w.dtype == TVB_I8_TENSOR, "prefill: weight dtype %d", (int)w.dtype);
    const size_t n = (size_t)rows * K;
    if (!c->pf_w16) {
        // the largest projection group of a layer: gate + up, q + k + v, o or down
        const size_t need = std::max({(size_t)2 * c->I * c->H, (size_t)(c->Hq + 2 * c->Hk) * c->H,
                                      (size_t)c->H * c->Hq, (size_t)c->H * c->I});
        TVB_TRY(alloc_dev((void**)&c->pf_w16, need * 2));
        c->pf_w16_elems = need;
    }
    TVB_REQUIRE(off + n <= c->pf_w16_elems, "prefill: INT8 widening scratch too small");
    TVB_TRY(pf_i8_to_f16(static_cast<const int8_t*>(w.w), n, c->pf_w16 + off, c->stream, pdl));
    m.w = c->pf_w16 + off;
    off += n;
    if (w.dtype == TVB_I8_ROW) m.row_scales = w.row_scales;
    else m.scale = w.tensor_scale;
    return TVB_OK;
}

// The prompt in chunks of the workspace's rows: per layer RMSNorm -> q/k/v on
// the tensor cores with RoPE and KV append fused -> causal attention over every
// KV row so far -> sub-norm -> o_proj + residual -> ffn_norm -> gate/up with
// relu^2 * up fused -> sub-norm -> down + residual; then output_norm + lm_head
// + argmax of the last row, leaving the step state at (pos S, argmax).
//
// Tensor parallelism: q/k/v, attention and gate/up run on this rank's heads and
// rows; o_proj and down multiply this rank's columns into its exchange region
// (the sub-norm before them deferred to the reduction), and after a flag sync
// every rank adds all ranks' partial rows, in rank order, to its copy of the
// residual.  The lm_head takes this rank's vocabulary slice and the ranks agree
// on the argmax through the decode step's key exchange.
// Scoring job of tvb_score_logprobs: after the layers of each prompt chunk, the
// rows that predict a scored token get their logits (output norm + tied
// lm_head, up to kLpRows at a time) and their log-probabilities.
struct LpJob {
    int first;          // first scored position (row first - 1 predicts it)
    int k;
    const int* target;  // device: the scored tokens, tokens[first ..]
    float* logits;      // device [kLpRows][V]
    float* lp;          // device [n]
    int* ids;           // device [n][k]
    float* top;         // device [n][k]
};
constexpr int kLpRows = 64;

tvb_status prefill_batched(tvb_context* c, const int* tokens, int S, int slot, const LpJob* job = nullptr) {
    TVB_TRY(pf_workspace(c));
    float* const kslot = c->kcache + (size_t)slot * c->slot_floats;
    float* const vslot = c->vcache + (size_t)slot * c->slot_floats;
    const cudaStream_t st = c->stream;
    const int H = c->H, Hq = c->Hq, Hk = c->Hk, I = c->I, hd = c->cfg.head_dim;
    const float eps = c->cfg.rms_norm_eps, scale = 1.0f / std::sqrt((float)hd);
    const bool tp = c->tp_world > 1;
    TpArgs tpa = {};
    size_t reg_off[2] = {0, 0};
    float* reg[2] = {nullptr, nullptr};
    if (tp) {
        tpa.world = c->tp_world;
        tpa.rank = c->tp_rank;
        tpa.ld = H + 4;
        for (int r = 0; r < c->tp_world; ++r) tpa.peer[r] = c->tp_peer[r];
        tpa.index = -1;
        tpa.fold = -1;
        const size_t region = tp_prefill_region_floats(c->pf_cap, H);
        for (int j = 0; j < 2; ++j) {
            reg_off[j] = c->tp_pf_off + j * region;
            reg[j] = c->tp_xchg + reg_off[j];
        }
    }
    // a row-parallel projection: its partial rows into exchange region j, a
    // sync, and the residual += inv_rms * the ranks' partial rows
    auto exchange = [&](int j, int n, const void* sub_norm, int k_local) -> tvb_status {
        TVB_TRY(tp_sync(tpa, c->st, st));
        return tp_reduce_rows(tpa, reg_off[j], n, H, sub_norm ? k_local * c->tp_world : 0, eps, c->pf_x, st);
    };
    for (int i = 0; i < S; ++i) c->h_io[i] = tokens[i];
    TVB_CUDA(cudaMemcpyAsync(c->pf_tok, c->h_io, (size_t)S * 4, cudaMemcpyHostToDevice, st));
    int last_rows = 0;
    for (int p0 = 0; p0 < S; p0 += c->pf_cap) {
        const int n = std::min(c->pf_cap, S - p0);
        last_rows = n;
        TVB_TRY(pf_embed(static_cast<const uint16_t*>(c->tok_embd), c->pf_tok + p0, n, H, c->pf_x, st));
        for (int l = 0; l < c->L; ++l) {
            const tvb_layer_weights& lw = c->layers[l];
            float* kl = kslot + (size_t)l * c->cfg.max_seq_len * Hk;
            float* vl = vslot + (size_t)l * c->cfg.max_seq_len * Hk;
            size_t off = 0;
            PfGemm g;
            g.part = c->pf_part;
            g.flags = c->pf_flags;
            g.part_floats = c->pf_part_floats;
            g.S = n;
            g.xh = c->pf_xh;
            g.xl = c->pf_xl;
            g.row_exp = c->pf_exp;
            g.status = &c->st->status;
            // attn_norm -> q, k, v -> RoPE -> KV rows p0 ..
            TVB_TRY(pf_norm_split(c->pf_x, lw.attn_norm, n, H, eps, c->pf_xh, c->pf_xl, c->pf_exp, st));
            g.mode = PF_QKV;
            g.K = H;
            TVB_TRY(pf_operand(c, lw.wq, Hq, H, off, g.m[0]));
            TVB_TRY(pf_operand(c, lw.wk, Hk, H, off, g.m[1]));
            TVB_TRY(pf_operand(c, lw.wv, Hk, H, off, g.m[2]));
            g.nh = c->cfg.num_heads;
            g.nkv = c->cfg.num_kv_heads;
            g.hd = hd;
            g.pos0 = p0;
            g.q_out = c->pf_q;
            g.kcache = kl;
            g.vcache = vl;
            g.rope_cos = c->rope_cos;
            g.rope_sin = c->rope_sin;
            TVB_TRY(pf_gemm(g, st));
            if (c->pf_planes)
                TVB_TRY(pf_attention_tc(c->pf_q, kl, vl, n, p0, g.nh, g.nkv, hd, scale, c->pf_attn, c->pf_planes,
                                        c->pf_cap, c->cfg.max_seq_len, &c->st->status, st));
            else
                TVB_TRY(pf_attention(c->pf_q, kl, vl, n, p0, g.nh, g.nkv, hd, scale, c->pf_attn, st));
            // attn_sub_norm -> o_proj -> residual
            TVB_TRY(pf_norm_split(c->pf_attn, lw.attn_sub_norm, n, Hq, eps, c->pf_xh, c->pf_xl, c->pf_exp, st,
                                  tp ? reg[0] + (size_t)n * H : nullptr));
            off = 0;
            g.mode = tp ? PF_STORE : PF_RESID;
            g.K = Hq;
            TVB_TRY(pf_operand(c, lw.wo, H, Hq, off, g.m[0]));
            g.y = tp ? reg[0] : c->pf_x;
            g.ldy = H;
            TVB_TRY(pf_gemm(g, st));
            if (tp) TVB_TRY(exchange(0, n, lw.attn_sub_norm, Hq));
            // ffn_norm -> gate/up -> relu^2 * up
            TVB_TRY(pf_norm_split(c->pf_x, lw.ffn_norm, n, H, eps, c->pf_xh, c->pf_xl, c->pf_exp, st));
            off = 0;
            g.mode = PF_GATEUP;
            g.K = H;
            TVB_TRY(pf_operand(c, lw.w_gate, I, H, off, g.m[0]));
            TVB_TRY(pf_operand(c, lw.w_up, I, H, off, g.m[1]));
            g.y = c->pf_h;
            g.ldy = I;
            TVB_TRY(pf_gemm(g, st));
            // ffn_sub_norm -> down -> residual
            TVB_TRY(pf_norm_split(c->pf_h, lw.ffn_sub_norm, n, I, eps, c->pf_xh, c->pf_xl, c->pf_exp, st,
                                  tp ? reg[1] + (size_t)n * H : nullptr));
            off = 0;
            g.mode = tp ? PF_STORE : PF_RESID;
            g.K = I;
            TVB_TRY(pf_operand(c, lw.w_down, H, I, off, g.m[0]));
            g.y = tp ? reg[1] : c->pf_x;
            g.ldy = H;
            TVB_TRY(pf_gemm(g, st));
            if (tp) TVB_TRY(exchange(1, n, lw.ffn_sub_norm, I));
        }
        if (job) {
            // rows p0 + r predicting scored tokens: r in [first - 1 - p0, S - 1 - p0) of this chunk
            const int r0 = std::max(0, job->first - 1 - p0), r1 = std::min(n, S - 1 - p0);
            for (int a0 = r0; a0 < r1; a0 += kLpRows) {
                const int cnt = std::min(kLpRows, r1 - a0);
                const int j0 = p0 + a0 - (job->first - 1);   // index of the first scored token
                TVB_TRY(pf_norm_split(c->pf_x + (size_t)a0 * H, c->output_norm, cnt, H, eps, c->pf_xh, c->pf_xl,
                                      c->pf_exp, st));
                PfGemm lg;
                lg.mode = PF_STORE;
                lg.S = cnt;
                lg.K = H;
                lg.xh = c->pf_xh;
                lg.xl = c->pf_xl;
                lg.row_exp = c->pf_exp;
                lg.status = &c->st->status;
                lg.part = c->pf_part;
                lg.flags = c->pf_flags;
                lg.part_floats = c->pf_part_floats;
                lg.m[0].w = static_cast<const uint16_t*>(c->tok_embd);
                lg.m[0].rows = c->V;
                lg.y = job->logits;
                lg.ldy = c->V;
                TVB_TRY(pf_gemm(lg, st));
                TVB_TRY(logprob_rows(job->logits, cnt, c->V, c->V, job->target + j0, job->k, job->lp + j0,
                                     job->k ? job->ids + (size_t)j0 * job->k : nullptr,
                                     job->k ? job->top + (size_t)j0 * job->k : nullptr, st));
            }
        }
    }
    // output_norm + lm_head + argmax of the last row (the decode step's last
    // phase as a stand-alone launch); it advances the step state to (S, argmax)
    c->h_io[S] = S - 1;
    c->h_io[S + 1] = tokens[S - 1];
    TVB_CUDA(cudaMemcpyAsync(c->st, c->h_io + S, 8, cudaMemcpyHostToDevice, st));
    GemvArgs a = {};
    const int vs = c->V / c->tp_world;   // this rank's vocabulary slice
    a.w[0] = static_cast<const uint16_t*>(c->tok_embd) + (size_t)c->tp_rank * vs * H;
    a.tscale[0] = 1.0f;
    a.N = vs;
    a.K = H;
    a.x = c->pf_x + (size_t)(last_rows - 1) * H;
    a.norm_w = c->output_norm;
    a.eps = eps;
    a.y = c->e_logits;
    a.st = c->st;
    a.status = &c->st->status;
    if (!tp) return launch_gemv<GM_LMHEAD, WT_F16, 1>(a, st, false);
    a.tp = tpa;
    a.tp.vocab0 = c->tp_rank * vs;
    a.tp.index = 0;   // the argmax exchange over the ranks' slices
    return launch_gemv<GM_LMHEAD, WT_F16, 1, true>(a, st, false);
}

// One greedy step of B sequences (tvb_decode_batch): row b is sequence b (KV
// slot b) with token tokens[b] at position positions[b].  The layer sequence is
// the batched prefill's with one row per sequence: the GEMMs read every weight
// once for all B rows (split over K so the few rows keep the SMs streaming),
// RoPE and the KV append use each row's own position and slot, and attention
// runs per sequence over its slot.  Under tensor parallelism the row-parallel
// partials are exchanged as in the batched prefill and every rank takes the
// largest of the ranks' per-row argmax keys.  Leaves the B next tokens in
// h_io[2B ..) after the stream is synchronised, the logits of this rank's
// vocabulary slice in bd_logits [B][V / world].  The tokens and positions are
// read from the pinned staging h_io[0, 2B), so the step can be captured.
tvb_status decode_batch(tvb_context* c, int B) {
    const cudaStream_t st = c->stream;
    const int H = c->H, Hq = c->Hq, Hk = c->Hk, I = c->I, hd = c->cfg.head_dim;
    const float eps = c->cfg.rms_norm_eps, scale = 1.0f / std::sqrt((float)hd);
    const bool tp = c->tp_world > 1;
    // programmatic dependent launch between the step's kernels: each may start
    // (TMEM, barriers, weight requests) while its predecessor finishes
    const bool pdl = !g_disable_pdl;
    TpArgs tpa = {};
    size_t reg_off[2] = {0, 0};
    float* reg[2] = {nullptr, nullptr};
    if (tp) {
        tpa.world = c->tp_world;
        tpa.rank = c->tp_rank;
        tpa.ld = H + 4;
        for (int r = 0; r < c->tp_world; ++r) tpa.peer[r] = c->tp_peer[r];
        tpa.index = -1;
        tpa.fold = -1;
        const size_t region = tp_prefill_region_floats(c->pf_cap, H);
        for (int j = 0; j < 2; ++j) {
            reg_off[j] = c->tp_pf_off + j * region;
            reg[j] = c->tp_xchg + reg_off[j];
        }
    }
    auto exchange = [&](int j, const void* sub_norm, int k_local) -> tvb_status {
        TVB_TRY(tp_sync(tpa, c->st, st, pdl));
        return tp_reduce_rows(tpa, reg_off[j], B, H, sub_norm ? k_local * c->tp_world : 0, eps, c->pf_x, st, pdl);
    };
    int* d_tok = c->bd_io;
    int* d_pos = c->bd_io + kMaxBatch;
    int* d_next = c->bd_io + 2 * kMaxBatch;
    TVB_CUDA(cudaMemcpyAsync(d_tok, c->h_io, (size_t)B * 4, cudaMemcpyHostToDevice, st));
    TVB_CUDA(cudaMemcpyAsync(d_pos, c->h_io + B, (size_t)B * 4, cudaMemcpyHostToDevice, st));
    TVB_TRY(pf_embed(static_cast<const uint16_t*>(c->tok_embd), d_tok, B, H, c->pf_x, st, pdl));
    // attention splits: enough (kv head, split, sequence) CTAs to cover the SMs
    const int nkv = c->cfg.num_kv_heads;
    const int nsplit = std::max(1, std::min(kMaxAttnSplits, (num_sms() + nkv * B - 1) / (nkv * B)));
    for (int l = 0; l < c->L; ++l) {
        const tvb_layer_weights& lw = c->layers[l];
        float* kl = c->kcache + (size_t)l * c->cfg.max_seq_len * Hk;   // slot 0; row b adds b slots
        float* vl = c->vcache + (size_t)l * c->cfg.max_seq_len * Hk;
        size_t off = 0;
        PfGemm g;
        g.S = B;
        g.xh = c->pf_xh;
        g.xl = c->pf_xl;
        g.row_exp = c->pf_exp;
        g.status = &c->st->status;
        g.part = c->pf_part;
        g.flags = c->pf_flags;
        g.part_floats = c->pf_part_floats;
        g.pdl = pdl;
        // attn_norm -> q, k, v -> RoPE at each row's position -> KV slot rows
        TVB_TRY(pf_norm_split(c->pf_x, lw.attn_norm, B, H, eps, c->pf_xh, c->pf_xl, c->pf_exp, st, nullptr, pdl));
        g.mode = PF_QKV;
        g.K = H;
        TVB_TRY(pf_operand(c, lw.wq, Hq, H, off, g.m[0], pdl));
        TVB_TRY(pf_operand(c, lw.wk, Hk, H, off, g.m[1], pdl));
        TVB_TRY(pf_operand(c, lw.wv, Hk, H, off, g.m[2], pdl));
        g.nh = c->cfg.num_heads;
        g.nkv = nkv;
        g.hd = hd;
        g.q_out = c->pf_q;
        g.kcache = kl;
        g.vcache = vl;
        g.rope_cos = c->rope_cos;
        g.rope_sin = c->rope_sin;
        g.row_pos = d_pos;
        g.kv_slot_stride = c->slot_floats;
        TVB_TRY(pf_gemm(g, st));
        g.row_pos = nullptr;
        TVB_TRY(batch_attention(c->pf_q, kl, vl, c->slot_floats, d_pos, B, g.nh, nkv, hd, nsplit, scale,
                                c->bd_attn_part, c->pf_attn, st, pdl));
        // attn_sub_norm -> o_proj -> residual
        TVB_TRY(pf_norm_split(c->pf_attn, lw.attn_sub_norm, B, Hq, eps, c->pf_xh, c->pf_xl, c->pf_exp, st,
                              tp ? reg[0] + (size_t)B * H : nullptr, pdl));
        off = 0;
        g.mode = tp ? PF_STORE : PF_RESID;
        g.K = Hq;
        TVB_TRY(pf_operand(c, lw.wo, H, Hq, off, g.m[0], pdl));
        g.y = tp ? reg[0] : c->pf_x;
        g.ldy = H;
        TVB_TRY(pf_gemm(g, st));
        if (tp) TVB_TRY(exchange(0, lw.attn_sub_norm, Hq));
        // ffn_norm -> gate/up -> relu^2 * up
        TVB_TRY(pf_norm_split(c->pf_x, lw.ffn_norm, B, H, eps, c->pf_xh, c->pf_xl, c->pf_exp, st, nullptr, pdl));
        off = 0;
        g.mode = PF_GATEUP;
        g.K = H;
        TVB_TRY(pf_operand(c, lw.w_gate, I, H, off, g.m[0], pdl));
        TVB_TRY(pf_operand(c, lw.w_up, I, H, off, g.m[1], pdl));
        g.y = c->pf_h;
        g.ldy = I;
        TVB_TRY(pf_gemm(g, st));
        // ffn_sub_norm -> down -> residual
        TVB_TRY(pf_norm_split(c->pf_h, lw.ffn_sub_norm, B, I, eps, c->pf_xh, c->pf_xl, c->pf_exp, st,
                              tp ? reg[1] + (size_t)B * H : nullptr, pdl));
        off = 0;
        g.mode = tp ? PF_STORE : PF_RESID;
        g.K = I;
        TVB_TRY(pf_operand(c, lw.w_down, H, I, off, g.m[0], pdl));
        g.y = tp ? reg[1] : c->pf_x;
        g.ldy = H;
        TVB_TRY(pf_gemm(g, st));
        if (tp) TVB_TRY(exchange(1, lw.ffn_sub_norm, I));
    }
    // output_norm + tied lm_head over this rank's vocabulary slice, then the
    // per-row greedy argmax (model.cpp:1571-1580 per sequence)
    const int vs = c->V / c->tp_world;
    TVB_TRY(pf_norm_split(c->pf_x, c->output_norm, B, H, eps, c->pf_xh, c->pf_xl, c->pf_exp, st, nullptr, pdl));
    PfGemm g;
    g.mode = PF_STORE;
    g.S = B;
    g.K = H;
    g.xh = c->pf_xh;
    g.xl = c->pf_xl;
    g.row_exp = c->pf_exp;
    g.status = &c->st->status;
    g.part = c->pf_part;
    g.flags = c->pf_flags;
    g.part_floats = c->pf_part_floats;
    g.pdl = pdl;
    g.m[0].w = static_cast<const uint16_t*>(c->tok_embd) + (size_t)c->tp_rank * vs * H;
    g.m[0].rows = vs;
    g.y = c->bd_logits;
    g.ldy = vs;
    TVB_TRY(pf_gemm(g, st));
    KeySources src = {};
    if (tp) {
        // every rank publishes its B keys in its own buffer, then takes the
        // largest over the ranks (the next step's syncs order the reuse)
        unsigned long long* own = reinterpret_cast<unsigned long long*>(c->tp_xchg + c->tp_key_off);
        TVB_TRY(batch_argmax(c->bd_logits, B, vs, vs, c->tp_rank * vs, own, st, pdl));
        TVB_TRY(tp_sync(tpa, c->st, st, pdl));
        src.n = c->tp_world;
        for (int r = 0; r < c->tp_world; ++r)
            src.p[r] = reinterpret_cast<const unsigned long long*>(c->tp_peer[r] + c->tp_key_off);
    } else {
        TVB_TRY(batch_argmax(c->bd_logits, B, vs, vs, 0, c->bd_keys, st, pdl));
        src.n = 1;
        src.p[0] = c->bd_keys;
    }
    TVB_TRY(batch_pick(src, B, d_next, st, pdl));
    TVB_CUDA(cudaMemcpyAsync(c->h_io + 2 * B, d_next, (size_t)B * 4, cudaMemcpyDeviceToHost, st));
    return TVB_OK;
}

}  // namespace

extern "C" {

tvb_status tvb_context_create(const tvb_model_config* cfg, tvb_context** out) {
    TVB_REQUIRE(cfg && out, "context_create: null argument");
    *out = nullptr;
    const tvb_model_config& m = *cfg;
    TVB_REQUIRE(m.hidden_size > 0 && m.num_layers > 0 && m.num_heads > 0 && m.num_kv_heads > 0 &&
                    m.intermediate_size > 0 && m.vocab_size > 0 && m.max_seq_len > 0,
                "context_create: non-positive dimension");
    TVB_REQUIRE(m.head_dim == 128, "context_create: head_dim %d (only 128 is built)", m.head_dim);
    TVB_REQUIRE(m.num_heads % m.num_kv_heads == 0, "context_create: heads %% kv_heads != 0");
    TVB_REQUIRE(m.num_kv_heads <= kMaxKvHeads, "context_create: too many kv heads");
    TVB_REQUIRE(m.hidden_size % 16 == 0 && m.intermediate_size % 16 == 0,
                "context_create: hidden/intermediate must be multiples of 16");
    {
        tvb_status ps = prepare_kernels();
        if (ps != TVB_OK) return ps;
        const char* e = std::getenv("TVB_DISABLE_PDL");
        g_disable_pdl = e && e[0] == '1';
    }
    tvb_context* c = new (std::nothrow) tvb_context();
    if (!c) return set_error(TVB_ERR_OOM, "context_create: host allocation");
    c->cfg = m;
    if (c->cfg.max_prefill <= 0) c->cfg.max_prefill = 1024;
    c->H = m.hidden_size;
    c->Hq = m.num_heads * m.head_dim;
    c->Hk = m.num_kv_heads * m.head_dim;
    c->I = m.intermediate_size;
    c->V = m.vocab_size;
    c->L = m.num_layers;
    c->nsplit = std::max(1, std::min(kMaxAttnSplits, num_sms() / m.num_kv_heads));
    c->layers.assign(c->L, tvb_layer_weights{});
    c->layer_set.assign(c->L, false);
    cudaGetDevice(&c->device);
    auto fail = [&](tvb_status s) {
        tvb_context_destroy(c);
        return s;
    };
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess)
        return fail(cuda_error(cudaGetLastError(), "cudaStreamCreate"));
    const int H = c->H, Hq = c->Hq, Hk = c->Hk, I = c->I, V = c->V;
    c->slots = std::max(1, m.max_batch);
    c->slot_floats = (size_t)c->L * m.max_seq_len * Hk;
    const size_t kv = c->slot_floats * c->slots;
    struct { void** p; size_t b; } allocs[] = {
        {(void**)&c->d_x, H * 4ull}, {(void**)&c->d_norm, std::max(H, I) * 4ull},
        {(void**)&c->d_q, Hq * 4ull}, {(void**)&c->d_k, Hk * 4ull}, {(void**)&c->d_v, Hk * 4ull},
        {(void**)&c->d_gate, I * 4ull}, {(void**)&c->d_up, I * 4ull},
        {(void**)&c->e_x, H * 4ull}, {(void**)&c->e_x2, H * 4ull}, {(void**)&c->e_q, Hq * 4ull},
        {(void**)&c->e_attn, Hq * 4ull},
        {(void**)&c->e_h, I * 4ull}, {(void**)&c->e_logits, V * 4ull},
        {(void**)&c->attn_part, (size_t)m.num_heads * 32 * (m.head_dim + 4) * 4ull},
        {(void**)&c->kcache, kv * 4}, {(void**)&c->vcache, kv * 4},
        {(void**)&c->rope_cos, (size_t)m.max_seq_len * (m.head_dim / 2) * 4},
        {(void**)&c->rope_sin, (size_t)m.max_seq_len * (m.head_dim / 2) * 4},
        {(void**)&c->st, sizeof(StepState)}, {(void**)&c->hist, (size_t)m.max_seq_len * 4},
    };
    for (auto& a : allocs) {
        tvb_status s = alloc_dev(a.p, a.b);
        if (s != TVB_OK) return fail(s);
    }
    struct { void** p; size_t b; } pins[] = {
        {(void**)&c->h_qkv, (Hq + 2ull * Hk) * 4}, {(void**)&c->h_attn, std::max(H, Hq) * 4ull},
        {(void**)&c->h_logit, V * 4ull}, {(void**)&c->h_st, sizeof(StepState)},
        {(void**)&c->h_io, (size_t)m.max_seq_len * 8}, {(void**)&c->h_hist, (size_t)m.max_seq_len * 4},
    };
    for (auto& a : pins) {
        cudaError_t e = cudaMallocHost(a.p, a.b);
        if (e != cudaSuccess) return fail(cuda_error(e, "cudaMallocHost"));
    }
    // RoPE factors with the CPU formulas (tensor.cpp:830-838), once per context.
    {
        const int half = m.head_dim / 2;
        std::vector<float> cs((size_t)m.max_seq_len * half), sn((size_t)m.max_seq_len * half);
        for (int p = 0; p < m.max_seq_len; ++p)
            for (int ic = 0; ic < half; ++ic) {
                float freq = 1.0f / std::pow(m.rope_theta, (float)(2 * ic) / (float)m.head_dim);
                cs[(size_t)p * half + ic] = std::cos(p * freq);
                sn[(size_t)p * half + ic] = std::sin(p * freq);
            }
        if (cudaMemcpy(c->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(c->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(cuda_error(cudaGetLastError(), "rope table upload"));
    }
    if (cudaMemset(c->st, 0, sizeof(StepState)) != cudaSuccess ||
        cudaMemset(c->kcache, 0, kv * 4) != cudaSuccess || cudaMemset(c->vcache, 0, kv * 4) != cudaSuccess)
        return fail(cuda_error(cudaGetLastError(), "context memset"));
    std::memset(c->h_st, 0, sizeof(StepState));
    *out = c;
    return TVB_OK;
}

tvb_status tvb_context_destroy(tvb_context* c) {
    if (!c) return TVB_OK;
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->g_step) cudaGraphExecDestroy(c->g_step);
    if (c->g_layers) cudaGraphExecDestroy(c->g_layers);
    if (c->bd_graph) cudaGraphExecDestroy(c->bd_graph);
    void* dev[] = {c->d_x, c->d_norm, c->d_q, c->d_k, c->d_v, c->d_gate, c->d_up, c->e_x, c->e_q,
                   c->e_attn, c->e_h, c->e_logits, c->attn_part, c->kcache, c->vcache,
                   c->rope_cos, c->rope_sin, c->st, c->hist, c->d_phases,
                   c->pf_x, c->pf_q, c->pf_attn, c->pf_h, c->pf_xh, c->pf_xl, c->pf_exp, c->pf_tok,
                   c->pf_w16, c->e_x2, c->tp_xchg, c->pf_planes, c->pf_inv, c->pf_part, c->pf_flags, c->bd_attn_part,
                   c->bd_logits, c->bd_io, c->bd_keys};
    for (void* p : dev)
        if (p) cudaFree(p);
    void* pin[] = {c->h_qkv, c->h_attn, c->h_logit, c->h_st, c->h_io, c->h_hist};
    for (void* p : pin)
        if (p) cudaFreeHost(p);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return TVB_OK;
}

void* tvb_context_stream(tvb_context* c) { return c ? (void*)c->stream : nullptr; }

tvb_status tvb_tp_init(tvb_context* c, int rank, int world, void** exchange) {
    TVB_REQUIRE(c && exchange, "tp_init: null argument");
    TVB_REQUIRE(world >= 1 && world <= kMaxTp && rank >= 0 && rank < world,
                "tp_init: rank %d of %d (at most %d ranks)", rank, world, kMaxTp);
    TVB_REQUIRE(c->V % world == 0, "tp_init: vocabulary %d not divisible by %d ranks", c->V, world);
    TVB_REQUIRE(!c->tp_xchg, "tp_init: already initialised");
    TVB_REQUIRE(num_sms() <= kTpMaxGrid, "tp_init: %d SMs, the exchange flags hold %d CTAs", num_sms(), kTpMaxGrid);
    // decode exchange area, then the batched-prefill region (partial rows and
    // row sums of squares of up to max_prefill rows)
    const size_t slots_end = (size_t)kTpSlots + 2ull * world * (c->H + 4);
    c->tp_xf_off = (slots_end + 63) / 64 * 64;   // row-exchange flags, [world][kTpMaxGrid]
    const size_t decode_floats = c->tp_xf_off + (size_t)world * kTpMaxGrid;
    c->tp_pf_off = (decode_floats + 63) / 64 * 64;
    const int pf_rows = std::min(c->cfg.max_prefill, c->cfg.max_seq_len);
    c->tp_key_off = c->tp_pf_off + 2 * tp_prefill_region_floats(pf_rows, c->H);
    const size_t floats = c->tp_key_off + 2 * kMaxBatch;   // + the batched step's argmax keys (u64)
    TVB_TRY(alloc_dev((void**)&c->tp_xchg, floats * 4));
    TVB_CUDA(cudaMemset(c->tp_xchg, 0, floats * 4));
    c->tp_world = world;
    c->tp_rank = rank;
    c->tp_ready = world == 1;
    if (world == 1) c->tp_peer[0] = c->tp_xchg;
    c->dirty = true;
    ++c->gen;
    *exchange = c->tp_xchg;
    return TVB_OK;
}

tvb_status tvb_tp_recover(tvb_context* c) {
    TVB_REQUIRE(c, "tp_recover: null context");
    TVB_REQUIRE(c->tp_xchg, "tp_recover: call tvb_tp_init first");
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    TVB_CUDA(cudaMemsetAsync(c->tp_xchg, 0, (c->tp_key_off + 2 * kMaxBatch) * 4, c->stream));
    TVB_CUDA(cudaMemsetAsync(c->st, 0, sizeof(StepState), c->stream));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    c->tp_failed = false;
    return TVB_OK;
}

tvb_status tvb_tp_set_peers(tvb_context* c, void* const* exchanges) {
    TVB_REQUIRE(c && exchanges, "tp_set_peers: null argument");
    TVB_REQUIRE(c->tp_xchg, "tp_set_peers: call tvb_tp_init first");
    TVB_REQUIRE(exchanges[c->tp_rank] == c->tp_xchg, "tp_set_peers: entry %d is not this rank's buffer",
                c->tp_rank);
    for (int r = 0; r < c->tp_world; ++r) {
        TVB_REQUIRE(exchanges[r] && (reinterpret_cast<uintptr_t>(exchanges[r]) & 15) == 0,
                    "tp_set_peers: bad buffer for rank %d", r);
        c->tp_peer[r] = static_cast<float*>(exchanges[r]);
    }
    c->tp_ready = true;
    c->dirty = true;
    ++c->gen;
    return TVB_OK;
}

tvb_status tvb_ipc_export(const void* dev_ptr, tvb_ipc_handle* out) {
    TVB_REQUIRE(dev_ptr && out, "ipc_export: null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(out->bytes), "IPC handle size");
    cudaIpcMemHandle_t h;
    TVB_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
    std::memcpy(out->bytes, &h, sizeof(h));
    return TVB_OK;
}

tvb_status tvb_ipc_import(const tvb_ipc_handle* in, void** dev_ptr) {
    TVB_REQUIRE(in && dev_ptr, "ipc_import: null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, in->bytes, sizeof(h));
    TVB_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return TVB_OK;
}

tvb_status tvb_ipc_close(void* dev_ptr) {
    TVB_REQUIRE(dev_ptr, "ipc_close: null argument");
    TVB_CUDA(cudaIpcCloseMemHandle(dev_ptr));
    return TVB_OK;
}

tvb_status tvb_context_buffers(tvb_context* c, tvb_buffers* o) {
    TVB_REQUIRE(c && o, "context_buffers: null argument");
    *o = tvb_buffers{c->d_x, c->d_norm, c->d_q, c->d_k, c->d_v, c->d_gate, c->d_up,
                     c->h_qkv, c->h_attn, c->h_logit};
    return TVB_OK;
}

tvb_status tvb_kv_clear(tvb_context* c) {
    TVB_REQUIRE(c, "kv_clear: null context");
    const size_t b = c->slot_floats * c->slots * 4;   // every slot
    TVB_CUDA(cudaMemsetAsync(c->kcache, 0, b, c->stream));
    TVB_CUDA(cudaMemsetAsync(c->vcache, 0, b, c->stream));
    return TVB_OK;
}

int tvb_kv_capacity(tvb_context* c) { return c ? c->cfg.max_seq_len : 0; }

tvb_status tvb_kv_layer_ptrs(tvb_context* c, int layer, float** k, float** v) {
    TVB_REQUIRE(c && k && v, "kv_layer_ptrs: null argument");
    TVB_REQUIRE(layer >= 0 && layer < c->L, "kv_layer_ptrs: layer %d", layer);
    *k = c->kcache + (size_t)layer * c->cfg.max_seq_len * c->Hk;
    *v = c->vcache + (size_t)layer * c->cfg.max_seq_len * c->Hk;
    return TVB_OK;
}

tvb_status tvb_kv_upload_layer(tvb_context* c, int layer, int n, const float* hk, const float* hv) {
    TVB_REQUIRE(c && hk && hv, "kv_upload_layer: null argument");
    TVB_REQUIRE(layer >= 0 && layer < c->L, "kv_upload_layer: layer %d", layer);
    if (n <= 0) return TVB_OK;
    n = std::min(n, c->cfg.max_seq_len);
    float *k, *v;
    tvb_kv_layer_ptrs(c, layer, &k, &v);
    TVB_CUDA(cudaMemcpyAsync(k, hk, (size_t)n * c->Hk * 4, cudaMemcpyHostToDevice, c->stream));
    TVB_CUDA(cudaMemcpyAsync(v, hv, (size_t)n * c->Hk * 4, cudaMemcpyHostToDevice, c->stream));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    return TVB_OK;
}

tvb_status tvb_kv_download_slot(tvb_context* c, int layer, int pos, int n_floats, float* dst) {
    TVB_REQUIRE(c && dst, "kv_download_slot: null argument");
    TVB_REQUIRE(layer >= 0 && layer < c->L && pos >= 0 && pos < c->cfg.max_seq_len,
                "kv_download_slot: layer %d pos %d", layer, pos);
    TVB_REQUIRE(n_floats >= 0 && n_floats <= c->Hk, "kv_download_slot: n_floats %d", n_floats);
    float *k, *v;
    tvb_kv_layer_ptrs(c, layer, &k, &v);
    TVB_CUDA(cudaMemcpyAsync(dst, k + (size_t)pos * c->Hk, (size_t)n_floats * 4, cudaMemcpyDeviceToHost,
                             c->stream));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    return TVB_OK;
}

tvb_status tvb_context_sync(tvb_context* c) {
    TVB_REQUIRE(c, "context_sync: null context");
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    return TVB_OK;
}

tvb_status tvb_trace_set(void* dev_buf, int n_phases) {
#ifdef TVB_PHASE_TRACE
    TVB_REQUIRE(n_phases >= 0, "trace_set: n_phases < 0");
    unsigned long long* p = static_cast<unsigned long long*>(dev_buf);
    TVB_CUDA(cudaMemcpyToSymbol(g_trace_buf, &p, sizeof(p)));
    TVB_CUDA(cudaMemcpyToSymbol(g_trace_phases, &n_phases, sizeof(n_phases)));
    return TVB_OK;
#else
    (void)dev_buf;
    (void)n_phases;
    return set_error(TVB_ERR_UNSUPPORTED, "trace_set: this build records no phase trace (libtvb200_trace.so does)");
#endif
}

tvb_status tvb_set_layer(tvb_context* c, int layer, const tvb_layer_weights* lw) {
    TVB_REQUIRE(c && lw, "set_layer: null argument");
    TVB_REQUIRE(layer >= 0 && layer < c->L, "set_layer: layer %d of %d", layer, c->L);
    const tvb_weight* ws[] = {&lw->wq, &lw->wk, &lw->wv, &lw->wo, &lw->w_gate, &lw->w_up, &lw->w_down};
    int wt0 = -1;
    for (const tvb_weight* w : ws) {
        int wt;
        TVB_REQUIRE(w->w, "set_layer %d: null weight", layer);
        TVB_REQUIRE(wt_of(w->dtype, &wt), "set_layer %d: dtype %d not a weight type", layer, (int)w->dtype);
        TVB_REQUIRE(w->dtype != TVB_I8_ROW || w->row_scales, "set_layer %d: TVB_I8_ROW needs row_scales", layer);
        TVB_REQUIRE((reinterpret_cast<uintptr_t>(w->w) & 15) == 0, "set_layer %d: weights must be 16-byte aligned", layer);
        if (wt0 < 0) wt0 = wt;
        TVB_REQUIRE(wt == wt0, "set_layer %d: mixed F16/INT8 projections in one layer", layer);
    }
    TVB_REQUIRE(lw->attn_norm && lw->ffn_norm, "set_layer %d: missing norm weights", layer);
    c->layers[layer] = *lw;
    c->layer_set[layer] = true;
    c->dirty = true;
    ++c->gen;
    return TVB_OK;
}

tvb_status tvb_set_output(tvb_context* c, const void* tok_embd, const float* output_norm) {
    TVB_REQUIRE(c && tok_embd && output_norm, "set_output: null argument");
    TVB_REQUIRE((reinterpret_cast<uintptr_t>(tok_embd) & 15) == 0, "set_output: tok_embd must be 16-byte aligned");
    c->tok_embd = tok_embd;
    c->output_norm = output_norm;
    c->dirty = true;
    ++c->gen;
    return TVB_OK;
}

tvb_status tvb_decode_step(tvb_context* c, int token, int pos, float* logits_host, int* argmax_host) {
    TVB_REQUIRE(c, "decode_step: null context");
    TVB_TRY(tp_guard(c, "decode_step"));
    TVB_REQUIRE(token >= 0 && token < c->V, "decode_step: token %d outside vocab %d", token, c->V);
    TVB_REQUIRE(pos >= 0 && pos < c->cfg.max_seq_len, "decode_step: pos %d outside KV capacity %d", pos,
                c->cfg.max_seq_len);
    TVB_TRY(ensure_graphs(c));
    c->h_io[0] = pos;
    c->h_io[1] = token;
    TVB_CUDA(cudaMemcpyAsync(c->st, c->h_io, 8, cudaMemcpyHostToDevice, c->stream));
    TVB_CUDA(cudaGraphLaunch(c->g_step, c->stream));
    TVB_CUDA(cudaMemcpyAsync(c->h_st, c->st, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
    const size_t nl = (size_t)(c->V / c->tp_world);   // this rank's logits
    if (logits_host)
        TVB_CUDA(cudaMemcpyAsync(c->h_logit, c->e_logits, nl * 4, cudaMemcpyDeviceToHost, c->stream));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    TVB_TRY(check_status(c));
    if (logits_host) std::memcpy(logits_host, c->h_logit, nl * 4);
    if (argmax_host) *argmax_host = c->h_st->next_token;
    return TVB_OK;
}

tvb_status tvb_generate_greedy(tvb_context* c, int token, int pos, int n_steps, int* tokens_host) {
    TVB_REQUIRE(c && tokens_host, "generate_greedy: null argument");
    TVB_TRY(tp_guard(c, "generate_greedy"));
    TVB_REQUIRE(token >= 0 && token < c->V, "generate_greedy: token %d", token);
    TVB_REQUIRE(pos >= 0 && n_steps >= 0 && pos + n_steps <= c->cfg.max_seq_len,
                "generate_greedy: positions [%d, %d) exceed KV capacity %d", pos, pos + n_steps,
                c->cfg.max_seq_len);
    if (!n_steps) return TVB_OK;
    TVB_TRY(ensure_graphs(c));
    c->h_io[0] = pos;
    c->h_io[1] = token;
    TVB_CUDA(cudaMemcpyAsync(c->st, c->h_io, 8, cudaMemcpyHostToDevice, c->stream));
    for (int i = 0; i < n_steps; ++i) {
        TVB_CUDA(cudaGraphLaunch(c->g_step, c->stream));
        TVB_CUDA(cudaMemcpyAsync(c->hist + pos + i, &c->st->next_token, 4, cudaMemcpyDeviceToDevice, c->stream));
    }
    TVB_CUDA(cudaMemcpyAsync(c->h_hist, c->hist + pos, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, c->stream));
    TVB_CUDA(cudaMemcpyAsync(c->h_st, c->st, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    TVB_TRY(check_status(c));
    std::memcpy(tokens_host, c->h_hist, (size_t)n_steps * 4);
    return TVB_OK;
}

tvb_status tvb_decode_enqueue(tvb_context* c, int token, int pos, int n_steps) {
    TVB_REQUIRE(c, "decode_enqueue: null context");
    TVB_TRY(tp_guard(c, "decode_enqueue"));
    TVB_REQUIRE(token >= 0 && token < c->V, "decode_enqueue: token %d", token);
    TVB_REQUIRE(pos >= 0 && n_steps >= 0 && pos + n_steps <= c->cfg.max_seq_len,
                "decode_enqueue: positions [%d, %d) exceed KV capacity %d", pos, pos + n_steps,
                c->cfg.max_seq_len);
    TVB_TRY(ensure_graphs(c));
    c->h_io[0] = pos;
    c->h_io[1] = token;
    TVB_CUDA(cudaMemcpyAsync(c->st, c->h_io, 8, cudaMemcpyHostToDevice, c->stream));
    for (int i = 0; i < n_steps; ++i) TVB_CUDA(cudaGraphLaunch(c->g_step, c->stream));
    return TVB_OK;
}

tvb_status tvb_prefill(tvb_context* c, const int* tokens, int S, float* last_logits, int* argmax_host) {
    return tvb_prefill_slot(c, 0, tokens, S, last_logits, argmax_host);
}

tvb_status tvb_prefill_slot(tvb_context* c, int slot, const int* tokens, int S, float* last_logits,
                            int* argmax_host) {
    TVB_REQUIRE(c && tokens, "prefill: null argument");
    TVB_TRY(tp_guard(c, "prefill"));
    TVB_REQUIRE(slot >= 0 && slot < c->slots, "prefill: slot %d of %d", slot, c->slots);
    TVB_REQUIRE(S > 0 && S <= c->cfg.max_seq_len, "prefill: S=%d outside (0, %d]", S, c->cfg.max_seq_len);
    for (int i = 0; i < S; ++i)
        TVB_REQUIRE(tokens[i] >= 0 && tokens[i] < c->V, "prefill: token[%d]=%d outside vocab", i, tokens[i]);
    TVB_TRY(ensure_graphs(c));
    // the pinned staging is about to be rewritten: let earlier copies from it finish
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    if (!pf_batched_supported(c)) {
        TVB_REQUIRE(slot == 0, "prefill: KV slots other than 0 need the batched (tensor-core) prefill");
        // shapes the tensor-core kernels do not tile: one decode-step launch
        // per prompt row; row s attends to KV rows [0, s] as in
        // forward_prefill (model.cpp:1084 kv_len = s + 1)
        for (int s = 0; s < S; ++s) {
            c->h_io[2 * s] = s;
            c->h_io[2 * s + 1] = tokens[s];
            TVB_CUDA(cudaMemcpyAsync(c->st, c->h_io + 2 * s, 8, cudaMemcpyHostToDevice, c->stream));
            TVB_CUDA(cudaGraphLaunch(s + 1 < S ? c->g_layers : c->g_step, c->stream));
        }
    } else {
        TVB_TRY(prefill_batched(c, tokens, S, slot));
    }
    TVB_CUDA(cudaMemcpyAsync(c->h_st, c->st, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
    const size_t nl = (size_t)(c->V / c->tp_world);   // this rank's logits
    if (last_logits)
        TVB_CUDA(cudaMemcpyAsync(c->h_logit, c->e_logits, nl * 4, cudaMemcpyDeviceToHost, c->stream));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    TVB_TRY(check_status(c));
    if (last_logits) std::memcpy(last_logits, c->h_logit, nl * 4);
    if (argmax_host) *argmax_host = c->h_st->next_token;
    return TVB_OK;
}

tvb_status tvb_score_logprobs(tvb_context* c, const int* tokens, int T, int start_pos, int k, float* logprobs,
                              int* top_ids, float* top_logprobs) {
    TVB_REQUIRE(c && tokens && logprobs, "score_logprobs: null argument");
    TVB_TRY(tp_guard(c, "score_logprobs"));
    TVB_REQUIRE(T > 0 && T <= c->cfg.max_seq_len, "score_logprobs: T=%d outside (0, %d]", T, c->cfg.max_seq_len);
    TVB_REQUIRE(k >= 0 && k <= kMaxLogprobsHost && (k == 0 || (top_ids && top_logprobs)),
                "score_logprobs: k=%d (0 .. %d, with output arrays)", k, kMaxLogprobsHost);
    TVB_REQUIRE(c->tp_world == 1, "score_logprobs: not built for tensor-parallel contexts");
    TVB_REQUIRE(pf_batched_supported(c), "score_logprobs: shapes the tensor-core GEMM does not tile");
    for (int i = 0; i < T; ++i)
        TVB_REQUIRE(tokens[i] >= 0 && tokens[i] < c->V, "score_logprobs: token[%d]=%d outside vocab", i, tokens[i]);
    const int first = std::max(1, start_pos);
    const int n = T - first;
    TVB_TRY(ensure_graphs(c));
    TVB_TRY(pf_workspace(c));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    if (n <= 0) return tvb_prefill(c, tokens, T, nullptr, nullptr);
    // per call: the scored tokens, one logits block, the results
    const size_t bytes = (size_t)n * 4 + (size_t)kLpRows * c->V * 4 + (size_t)n * 4 + (size_t)n * k * 8;
    char* ws = nullptr;
    TVB_CUDA(cudaMallocAsync((void**)&ws, bytes, c->stream));
    LpJob job;
    job.first = first;
    job.k = k;
    job.target = reinterpret_cast<const int*>(ws);
    job.logits = reinterpret_cast<float*>(ws + (size_t)n * 4);
    job.lp = job.logits + (size_t)kLpRows * c->V;
    job.ids = reinterpret_cast<int*>(job.lp + n);
    job.top = reinterpret_cast<float*>(job.ids + (size_t)n * k);
    tvb_status s = TVB_OK;
    if (cudaMemcpyAsync(ws, tokens + first, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        s = cuda_error(cudaGetLastError(), "score_logprobs: token upload");
    if (s == TVB_OK) s = prefill_batched(c, tokens, T, 0, &job);
    if (s == TVB_OK) {
        cudaMemcpyAsync(logprobs, job.lp, (size_t)n * 4, cudaMemcpyDeviceToHost, c->stream);
        if (k) {
            cudaMemcpyAsync(top_ids, job.ids, (size_t)n * k * 4, cudaMemcpyDeviceToHost, c->stream);
            cudaMemcpyAsync(top_logprobs, job.top, (size_t)n * k * 4, cudaMemcpyDeviceToHost, c->stream);
        }
    }
    cudaFreeAsync(ws, c->stream);
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    if (s != TVB_OK) return s;
    return check_status(c);
}

tvb_status tvb_decode_batch(tvb_context* c, const int* tokens, const int* positions, int B, float* logits,
                            int* next_tokens) {
    TVB_REQUIRE(c && tokens && positions && next_tokens, "decode_batch: null argument");
    TVB_TRY(tp_guard(c, "decode_batch"));
    TVB_REQUIRE(B >= 1 && B <= c->slots && B <= kMaxBatch && 3 * B <= 2 * c->cfg.max_seq_len,
                "decode_batch: B=%d (context slots %d, at most %d)", B, c->slots, kMaxBatch);
    for (int b = 0; b < B; ++b) {
        TVB_REQUIRE(tokens[b] >= 0 && tokens[b] < c->V, "decode_batch: token[%d]=%d outside vocab", b, tokens[b]);
        TVB_REQUIRE(positions[b] >= 0 && positions[b] < c->cfg.max_seq_len,
                    "decode_batch: position[%d]=%d outside [0, %d)", b, positions[b], c->cfg.max_seq_len);
    }
    TVB_REQUIRE(pf_batched_supported(c), "decode_batch: shapes the tensor-core GEMM does not tile");
    if (c->tp_world > 1) TVB_REQUIRE(c->tp_ready, "decode_batch: peers not set (tvb_tp_set_peers)");
    TVB_TRY(pf_workspace(c));
    TVB_CUDA(cudaStreamSynchronize(c->stream));   // the pinned staging is reused
    for (int b = 0; b < B; ++b) {
        c->h_io[b] = tokens[b];
        c->h_io[B + b] = positions[b];
    }
    // ~10 launches per layer: replayed as one graph once this batch size has
    // run eagerly (its lazy set-up done) under the current weights
    if (c->bd_gen != c->gen) {
        if (c->bd_graph) cudaGraphExecDestroy(c->bd_graph);
        c->bd_graph = nullptr;
        c->bd_eager = 0;
        c->bd_gen = c->gen;
    }
    const unsigned long long bit = 1ull << B;
    if (c->bd_graph && c->bd_graph_B == B) {
        TVB_CUDA(cudaGraphLaunch(c->bd_graph, c->stream));
    } else if (c->bd_eager & bit) {
        if (c->bd_graph) cudaGraphExecDestroy(c->bd_graph);
        c->bd_graph = nullptr;
        TVB_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        const tvb_status s = decode_batch(c, B);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(c->stream, &g);
        if (s != TVB_OK || e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return s != TVB_OK ? s : cuda_error(e, "cudaStreamEndCapture");
        }
        const cudaError_t ie = cudaGraphInstantiate(&c->bd_graph, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) return cuda_error(ie, "cudaGraphInstantiate (batched step)");
        c->bd_graph_B = B;
        TVB_CUDA(cudaGraphLaunch(c->bd_graph, c->stream));
    } else {
        TVB_TRY(decode_batch(c, B));
        c->bd_eager |= bit;
    }
    const int vs = c->V / c->tp_world;
    if (logits)
        TVB_CUDA(cudaMemcpyAsync(logits, c->bd_logits, (size_t)B * vs * 4, cudaMemcpyDeviceToHost, c->stream));
    TVB_CUDA(cudaMemcpyAsync(c->h_st, c->st, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
    TVB_CUDA(cudaStreamSynchronize(c->stream));
    TVB_TRY(check_status(c));
    for (int b = 0; b < B; ++b) next_tokens[b] = c->h_io[2 * B + b];
    return TVB_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Standalone device-pointer ops (the CUDABackend per-op API).
// ---------------------------------------------------------------------------
namespace tvb {

tvb_status standalone_gemv(float* y, const float* x, const void* W, int wt, const float* row_scales,
                           float tscale, int K, int N, cudaStream_t st) {
    TVB_REQUIRE(y && x && W, "gemv: null pointer");
    TVB_REQUIRE(K > 0 && N > 0, "gemv: bad shape K=%d N=%d", K, N);
    TVB_REQUIRE(wt == WT_F16 ? K % 8 == 0 : K % 16 == 0, "gemv: K=%d must be a multiple of %d", K,
                wt == WT_F16 ? 8 : 16);
    TVB_REQUIRE((reinterpret_cast<uintptr_t>(W) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
                "gemv: W and x must be 16-byte aligned");
    TVB_TRY(prepare_kernels());
    unsigned* status = nullptr;
    TVB_CUDA(cudaGetSymbolAddress((void**)&status, g_standalone_status));
    GemvArgs a = {};
    a.w[0] = W;
    a.row_scale[0] = row_scales;
    a.tscale[0] = tscale;
    a.N = N;
    a.K = K;
    a.x = x;
    a.y = y;
    a.status = status;
    return wt == WT_F16 ? launch_gemv<GM_PLAIN, WT_F16, 1>(a, st, false)
                        : launch_gemv<GM_PLAIN, WT_I8, 1>(a, st, false);
}

tvb_status standalone_attention(const float* q, const float* kc, const float* vc, int kv_len, float* out,
                                int nh, int nkv, int hd, float scale, cudaStream_t st) {
    TVB_REQUIRE(q && kc && vc && out, "attention: null pointer");
    TVB_REQUIRE(hd == 128, "attention: head_dim %d (only 128 is built)", hd);
    TVB_REQUIRE(nh > 0 && nkv > 0 && nh % nkv == 0, "attention: heads %d / kv heads %d", nh, nkv);
    TVB_REQUIRE(kv_len > 0, "attention: kv_len %d", kv_len);
    AttnArgs a = {};
    a.q = q;
    a.kcache = kc;
    a.vcache = vc;
    a.out = out;
    a.nh = nh;
    a.nkv = nkv;
    a.hd = hd;
    a.nsplit = 1;
    a.scale = scale;
    a.kv_len = kv_len;
    return launch_attn(a, st, false);
}

}  // namespace tvb
