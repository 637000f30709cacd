// tvq_session.cu -- device-resident executor for GPT-2-shaped stacks of
// QuantizedGemm layers (the tvq_session_* part of include/tvq.h).
//
// Replaces, for this path, InferenceSession.run -> ExecutionNode.execute ->
// the QuantizedGemm branch (tv/runtime/session.tkv:3403-3436, 678-697) and
// the initialize_weights upload (:3336-3350): weights are uploaded and
// quantized once, the whole forward (embedding, 4 INT8 linears per block,
// fp32 LayerNorm / attention / GELU, LM head) runs on one stream with no host
// round trip and is captured into a CUDA graph per batch layout.
//
// Per layer l the four activation quantization points use static per-tensor
// scales act_scale[4l + i] (i = 0 ln_1 output, 1 attention context, 2 ln_2
// output, 3 GELU output).  A calibration forward computes them on the GPU as
// calibrate_minmax would (tv/quantization/engine.tkv:13-36: scale =
// fl32(max(max|x|, 1e-8) / 127)), with the running max over calibration
// batches, and quantizes each activation with its own scale as it goes.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "tvq_common.cuh"
#include "tvq_glue.h"
#include "tvq_kernels.h"

namespace tvq {
namespace {

struct Lin {
    int8_t* W = nullptr;  // [n, k]
    float* sw = nullptr;  // [n]
    float* bias = nullptr;
    float* kvb = nullptr;  // c_attn, head dim 64: per-head K / V bounds (launch_kv_head_bound)
    int n = 0, k = 0;
    bool set = false;
};

struct LayerW {
    float* ln[4] = {nullptr, nullptr, nullptr, nullptr};  // ln_1 g, b, ln_2 g, b
    Lin lin[4];                                          // c_attn, attn c_proj, c_fc, mlp c_proj
};

struct Session {
    int device = 0;
    cudaStream_t st = nullptr;
    int vocab = 0, d = 0, heads = 0, layers = 0, ffn = 0, max_pos = 0, max_tokens = 0;
    double eps = 1e-6;
    std::vector<void*> allocs;
    float *wte = nullptr, *wpe = nullptr, *lnf_g = nullptr, *lnf_b = nullptr;
    // LM head operands split into fp16 high + low parts under power-of-two
    // row scales (launch_split_f16_rows)
    uint16_t *wte_hi = nullptr, *wte_lo = nullptr, *xf_hi = nullptr, *xf_lo = nullptr;
    float *wte_rs = nullptr, *xf_rs = nullptr;
    std::vector<LayerW> L;
    float* act_scale = nullptr;
    uint32_t* act_amax = nullptr;
    int64_t* ids = nullptr;
    int* seg = nullptr;
    int* tok_start = nullptr;
    int4* tiles = nullptr;   // attention work items {q0, seq start, seq end, 0}
    int4* split = nullptr;   // {key begin, key end, partial slot, 0}
    int4* comb = nullptr;    // partial merges {q0, seq end, first slot, count}
    float* part_o = nullptr;
    float2* part_ml = nullptr;
    int* counters = nullptr;  // per (merge entry, head): key-chunk partials counted in
    size_t tiles_cap = 0, split_cap = 0, comb_cap = 0, part_o_cap = 0, part_ml_cap = 0, counters_cap = 0;
    int ncomb = 0;
    bool attn_tc = false;  // head dim 64: tensor-core attention, 128-row query tiles
    int attn_rows = 64;
    // split Q, K and V^T, fp16 bits (tensor-core attention), and their head scales
    uint16_t *qh = nullptr, *ql = nullptr, *kh = nullptr, *kl = nullptr, *vh = nullptr, *vl = nullptr;
    int* kv_exp = nullptr;
    // exact int8 context: per layer and V column max |V| (written by c_attn),
    // the attention's fix-up list and its three counters (zero between launches)
    uint32_t* vmax = nullptr;
    int* fix_n = nullptr;       // rows, rows taken by the fix-up, finished fix-up CTAs
    int4* fix_list = nullptr;   // [fix_cap] rows with undecided int8 columns
    uint2* fix_mask = nullptr;  // [fix_cap] those columns
    int fix_cap = 0;
    float *x = nullptr, *qkv = nullptr, *hf = nullptr, *xf = nullptr, *xf_last = nullptr, *logits = nullptr;
    size_t logits_cap = 0;
    int8_t *aq = nullptr, *hq = nullptr;
    int* err = nullptr;
    // batch layout
    std::vector<int> seg_host;
    int T = 0, nseg = 0, ntiles = 0, logits_mode = 0;
    bool prepared = false;
    // captured graphs per mode (Mode below), rebuilt after prepare
    cudaGraphExec_t gexec[4] = {nullptr, nullptr, nullptr, nullptr};
    int64_t graph_kernels[4] = {0, 0, 0, 0};  // kernel nodes of each captured graph
    int last_mode = -1;                       // mode of the graph launched last
    int64_t extra_launches = 0;               // kernels launched beside that graph (LM head chunks)
    // host-bound logits: the copy stream and its events (created on first use)
    cudaStream_t cp = nullptr;
    std::vector<cudaEvent_t> chunk_ev;   // chunk c's logits are computed (on st)
    std::vector<cudaEvent_t> copied_ev;  // chunk c's rows have been copied out (on cp)
    cudaEvent_t copies_done = nullptr;   // every copy queued so far is done (on cp)
    // optional stage events recorded inside the captured graph (profiling)
    bool profile = false;
    std::vector<cudaEvent_t> ev;
    std::vector<int> ev_stage;  // stage id of the interval ending at ev[i]
    bool capturing = false;

    int64_t logits_rows() const { return logits_mode == 0 ? T : nseg; }

    void drop_graphs() {
        for (cudaGraphExec_t& g : gexec)
            if (g) {
                cudaGraphExecDestroy(g);
                g = nullptr;
            }
    }

    ~Session() {
        drop_graphs();
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
        for (cudaEvent_t e : chunk_ev) cudaEventDestroy(e);
        for (cudaEvent_t e : copied_ev) cudaEventDestroy(e);
        if (copies_done) cudaEventDestroy(copies_done);
        if (cp) cudaStreamDestroy(cp);
        for (void* p : allocs) cudaFree(p);
        if (st) cudaStreamDestroy(st);
    }
    template <typename T_>
    int alloc(T_** p, size_t count) {
        void* q = nullptr;
        cudaError_t e = cudaMalloc(&q, std::max<size_t>(count * sizeof(T_), 256));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (session)");
        allocs.push_back(q);
        *p = static_cast<T_*>(q);
        return TVQ_OK;
    }
};

std::mutex g_mu;
std::map<int64_t, std::unique_ptr<Session>> g_sessions;
int64_t g_next = 1;

Session* find(int64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_sessions.find(h);
    return it == g_sessions.end() ? nullptr : it->second.get();
}

// Makes the session's device current for the scope of one call.
struct DeviceGuard {
    int prev = -1;
    int rc = TVQ_OK;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaError_t e = cudaSetDevice(dev);
        if (e != cudaSuccess) rc = cuda_fail(e, "cudaSetDevice");
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

#define SESSION(h)                                                        \
    Session* S = find(h);                                                 \
    TVQ_CHECK(S, TVQ_ERR_HANDLE, "unknown or destroyed session handle");  \
    DeviceGuard dg__(S->device);                                          \
    if (dg__.rc) return dg__.rc;

#define STEP(expr)              \
    do {                        \
        int r__ = (expr);       \
        if (r__) return r__;    \
    } while (0)

void lin_shape(const Session& s, int which, int* n, int* k) {
    switch (which) {
        case 0: *n = 3 * s.d; *k = s.d; break;
        case 1: *n = s.d; *k = s.d; break;
        case 2: *n = s.ffn; *k = s.d; break;
        default: *n = s.d; *k = s.ffn; break;
    }
}

int gemm(Session& s, const int8_t* A, const Lin& l, const float* scale_a, float* Y, const float* residual,
         int8_t* Yq, const float* scale_out, uint32_t* amax, int act, bool kv_split = false,
         uint32_t* kv_vmax = nullptr) {
    GemmArgs g;
    if (kv_split) {  // c_attn on the tensor-core attention path: Q, K and V^T operands from the epilogue
        g.qh = s.qh;
        g.ql = s.ql;
        g.kh = s.kh;
        g.kl = s.kl;
        g.vth = s.vh;
        g.vtl = s.vl;
        g.kv_exp = s.kv_exp;
        g.kv_bound = l.kvb;
        // the f32 qkv is still written: the attention's exact fix-up of its
        // undecided int8 rows reads it, with the head maxima of V
        g.kv_vmax = kv_vmax;
        g.kvd = s.d;
        g.vt_pitch = attention_tc_pitch(s.T);
    }
    g.kind = GEMM_I8;
    g.A = A;
    g.W = l.W;
    g.bias = l.bias;
    g.residual = residual;
    g.Y = Y;
    g.Yq = Yq;
    g.m = s.T;
    g.n = l.n;
    g.k = l.k;
    g.scale_a = scale_a;
    g.scales_w = l.sw;
    g.per_channel = 1;
    g.act = act;
    g.scale_out = scale_out;
    g.amax = amax;
    return launch_gemm(g, s.st);
}

int attention(Session& s, int layer, float* out, int8_t* outq, const float* qscale, uint32_t* amax) {
    if (s.attn_tc) {  // K / V^T hi-lo come from the c_attn epilogue
        AttnFix fx;
        fx.vmax = s.vmax + static_cast<size_t>(layer) * s.d;
        fx.list = s.fix_list;
        fx.mask = s.fix_mask;
        fx.n = s.fix_n;
        fx.cap = s.fix_cap;
        return launch_attention_tc(s.qkv, s.qh, s.ql, s.kh, s.kl, s.vh, s.vl, s.kv_exp, s.T, s.tiles, s.split, s.ntiles, s.comb, s.ncomb,
                                   s.d, s.heads, out, outq, qscale, amax, s.part_o, s.part_ml, s.counters, s.st, &fx);
    }
    return launch_attention_split(s.qkv, s.tiles, s.split, s.ntiles, s.comb, s.ncomb, s.d, s.heads, out, outq, qscale,
                                  amax, s.part_o, s.part_ml, s.st);
}

// Stage ids reported by tvq_session_stage_times.
// ST_QUANT: the calibrate-then-quantize passes of a calibrating (dynamic)
// forward.
enum Stage { ST_EMBED = 0, ST_LN = 1, ST_GEMM_QKV = 2, ST_ATTN = 3, ST_GEMM_PROJ = 4, ST_GEMM_FC = 5, ST_GEMM_MPROJ = 6,
             ST_LM_HEAD = 7, ST_QUANT = 8, ST_COUNT = 9 };

// Marks the end of a stage inside the captured graph (profiling only).
int mark(Session& s, int stage) {
    if (!s.profile || !s.capturing) return TVQ_OK;
    cudaEvent_t e = nullptr;
    TVQ_CUDA(cudaEventCreate(&e));
    s.ev.push_back(e);
    s.ev_stage.push_back(stage);
    TVQ_CUDA(cudaEventRecordWithFlags(e, s.st, cudaEventRecordExternal));
    return TVQ_OK;
}

// What a captured graph runs: the whole forward (ids -> logits), the
// transformer blocks alone on the hidden states in s.x with static
// activation scales or with per-call (dynamic) calibration, or the forward up
// to the LM head's operand (M_BODY: the LM head then runs in row chunks
// whose logits are copied to the host while the next chunk computes).
enum Mode { M_FORWARD = 0, M_LAYERS = 1, M_LAYERS_DYNAMIC = 2, M_BODY = 3 };

// Rows of one LM-head chunk on the host-logits path (two 128-row tiles);
// TVQ_LOGIT_CHUNK_ROWS overrides it (a multiple of 128; 0 = one launch and
// one copy after it).
int logit_chunk_rows() {
    static const int rows = [] {
        const char* e = getenv("TVQ_LOGIT_CHUNK_ROWS");
        if (!e) return 256;
        const int v = atoi(e);
        return (v >= 0 && v % 128 == 0) ? v : 256;
    }();
    return rows;
}

// The transformer blocks on s.x (in place), enqueued on s.st.
int enqueue_layers(Session& s, bool calibrating) {
    const int T = s.T, d = s.d;
    if (s.attn_tc && s.ncomb > 0)  // merge counters start at 0 (a run that stopped early may leave them set)
        TVQ_CUDA(cudaMemsetAsync(s.counters, 0, sizeof(int) * static_cast<size_t>(s.ncomb) * s.heads, s.st));
    if (s.attn_tc)  // head maxima of V (atomicMax from c_attn) and the fix-up counters start at 0
        TVQ_CUDA(cudaMemsetAsync(s.vmax, 0, sizeof(uint32_t) * (static_cast<size_t>(s.layers) * s.d + 4), s.st));
    for (int l = 0; l < s.layers; l++) {
        LayerW& w = s.L[l];
        float* sc = s.act_scale + 4 * l;
        uint32_t* am = s.act_amax + 4 * l;
        // ln_1 -> int8 (c_attn input)
        if (calibrating) {
            STEP(launch_layernorm(s.x, w.ln[0], w.ln[1], s.hf, nullptr, nullptr, am + 0, T, d, s.eps, s.st));
            STEP(mark(s, ST_LN));
            STEP(launch_quantize_i8_amax(s.hf, s.aq, static_cast<int64_t>(T) * d, am + 0, sc + 0, s.st));
            STEP(mark(s, ST_QUANT));
        } else {
            STEP(launch_layernorm(s.x, w.ln[0], w.ln[1], nullptr, s.aq, sc + 0, nullptr, T, d, s.eps, s.st));
            STEP(mark(s, ST_LN));
        }
        // c_attn: qkv = dequant(aq Wqkv) + b
        STEP(gemm(s, s.aq, w.lin[0], sc + 0, s.qkv, nullptr, nullptr, nullptr, nullptr, TVQ_ACT_NONE, s.attn_tc,
                  s.vmax + static_cast<size_t>(l) * s.d));
        STEP(mark(s, ST_GEMM_QKV));
        // causal attention -> int8 context (attn c_proj input)
        if (calibrating) {
            STEP(attention(s, l, s.hf, nullptr, nullptr, am + 1));
            STEP(mark(s, ST_ATTN));
            STEP(launch_quantize_i8_amax(s.hf, s.aq, static_cast<int64_t>(T) * d, am + 1, sc + 1, s.st));
            STEP(mark(s, ST_QUANT));
        } else {
            STEP(attention(s, l, nullptr, s.aq, sc + 1, nullptr));
            STEP(mark(s, ST_ATTN));
        }
        // attn c_proj + residual, in place on x
        STEP(gemm(s, s.aq, w.lin[1], sc + 1, s.x, s.x, nullptr, nullptr, nullptr, TVQ_ACT_NONE));
        STEP(mark(s, ST_GEMM_PROJ));
        // ln_2 -> int8 (c_fc input)
        if (calibrating) {
            STEP(launch_layernorm(s.x, w.ln[2], w.ln[3], s.hf, nullptr, nullptr, am + 2, T, d, s.eps, s.st));
            STEP(mark(s, ST_LN));
            STEP(launch_quantize_i8_amax(s.hf, s.aq, static_cast<int64_t>(T) * d, am + 2, sc + 2, s.st));
            STEP(mark(s, ST_QUANT));
        } else {
            STEP(launch_layernorm(s.x, w.ln[2], w.ln[3], nullptr, s.aq, sc + 2, nullptr, T, d, s.eps, s.st));
            STEP(mark(s, ST_LN));
        }
        // c_fc + erf GELU -> int8 (mlp c_proj input)
        if (calibrating) {
            STEP(gemm(s, s.aq, w.lin[2], sc + 2, s.hf, nullptr, nullptr, nullptr, am + 3, TVQ_ACT_GELU_ERF));
            STEP(mark(s, ST_GEMM_FC));
            STEP(launch_quantize_i8_amax(s.hf, s.hq, static_cast<int64_t>(T) * s.ffn, am + 3, sc + 3, s.st));
            STEP(mark(s, ST_QUANT));
        } else {
            STEP(gemm(s, s.aq, w.lin[2], sc + 2, nullptr, nullptr, s.hq, sc + 3, nullptr, TVQ_ACT_GELU_ERF));
            STEP(mark(s, ST_GEMM_FC));
        }
        // mlp c_proj + residual, in place on x
        STEP(gemm(s, s.hq, w.lin[3], sc + 3, s.x, s.x, nullptr, nullptr, nullptr, TVQ_ACT_NONE));
        STEP(mark(s, ST_GEMM_MPROJ));
    }
    return TVQ_OK;
}

// Tied LM head on rows [r0, r0 + rows) of the split ln_f output, fp32 on the
// FP16 tensor cores with split precision (gpt2_ref.tkv:589-610): logits[r0:]
// of the same rows.  Rows are independent, so a chunk's logits are the
// same bits as those of a launch over all rows.
int launch_lm_head(Session& s, int r0, int rows, cudaStream_t st) {
    GemmArgs g;
    g.kind = GEMM_F16X3;
    g.A = s.xf_hi + static_cast<size_t>(r0) * s.d;
    g.A2 = s.xf_lo + static_cast<size_t>(r0) * s.d;
    g.W = s.wte_hi;
    g.W2 = s.wte_lo;
    g.scale_a = s.xf_rs + r0;
    g.scales_w = s.wte_rs;
    g.Y = s.logits + static_cast<size_t>(r0) * s.vocab;
    g.m = rows;
    g.n = s.vocab;
    g.k = s.d;
    g.per_channel = 0;
    return launch_gemm(g, st);
}

// The forward pass for the prepared layout, enqueued on s.st (without the LM
// head for M_BODY).
int enqueue_forward(Session& s, bool calibrating, bool lm_head = true) {
    const int T = s.T, d = s.d;
    STEP(mark(s, -1));
    STEP(launch_embed(s.ids, s.tok_start, s.wte, s.wpe, s.x, T, d, s.vocab, s.max_pos, s.err, s.st));
    STEP(mark(s, ST_EMBED));
    STEP(enqueue_layers(s, calibrating));
    // ln_f and the tied LM head (gpt2_ref.tkv:589-610), fp32; the LM head's
    // operand (row-scaled fp16 hi / lo) comes straight from ln_f for all rows
    int rows = T;
    if (s.logits_mode == 1) {
        STEP(launch_layernorm(s.x, s.lnf_g, s.lnf_b, s.xf, nullptr, nullptr, nullptr, T, d, s.eps, s.st));
        STEP(launch_gather_last(s.xf, s.seg, s.nseg, d, s.xf_last, s.st));
        rows = s.nseg;
        STEP(mark(s, ST_LN));
        STEP(launch_split_f16_rows(s.xf_last, s.xf_hi, s.xf_lo, s.xf_rs, rows, d, s.st));
    } else {
        STEP(launch_layernorm_split(s.x, s.lnf_g, s.lnf_b, s.xf_hi, s.xf_lo, s.xf_rs, T, d, s.eps, s.st));
        STEP(mark(s, ST_LN));
    }
    if (lm_head) {
        STEP(launch_lm_head(s, 0, rows, s.st));
        STEP(mark(s, ST_LM_HEAD));
    }
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

int check_ready(Session& s, bool layers_only = false) {
    TVQ_CHECK(layers_only || (s.vocab > 0 && s.wte && s.wpe && s.lnf_g && s.lnf_b), TVQ_ERR_INVALID,
              "embeddings / final layernorm not set");
    for (int l = 0; l < s.layers; l++) {
        for (int i = 0; i < 4; i++) TVQ_CHECK(s.L[l].ln[i], TVQ_ERR_INVALID, "layernorm not set");
        for (int i = 0; i < 4; i++) TVQ_CHECK(s.L[l].lin[i].set, TVQ_ERR_INVALID, "linear not set");
    }
    TVQ_CHECK(s.prepared, TVQ_ERR_INVALID, "tvq_session_prepare has not been called");
    return TVQ_OK;
}

int check_err(Session& s, cudaStream_t st) {
    TVQ_CUDA(cudaStreamSynchronize(st));
    int h = 0;
    TVQ_CUDA(cudaMemcpy(&h, s.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        TVQ_CUDA(cudaMemset(s.err, 0, sizeof(int)));
        set_error(TVQ_ERR_INVALID, "token id out of range or sequence longer than max_pos");
        return TVQ_ERR_INVALID;
    }
    return check_device_error(st);
}

int capture(Session& s, int mode) {
    if (s.profile) {
        // stage events belong to one graph at a time
        s.drop_graphs();
        for (cudaEvent_t e : s.ev) cudaEventDestroy(e);
        s.ev.clear();
        s.ev_stage.clear();
    } else if (s.gexec[mode]) {
        cudaGraphExecDestroy(s.gexec[mode]);
        s.gexec[mode] = nullptr;
    }
    cudaGraph_t g = nullptr;
    TVQ_CUDA(cudaStreamBeginCapture(s.st, cudaStreamCaptureModeRelaxed));
    s.capturing = true;
    int rc = TVQ_OK;
    if (mode == M_FORWARD || mode == M_BODY) {
        rc = enqueue_forward(s, false, mode == M_FORWARD);
    } else {
        rc = mark(s, -1);
        if (!rc && mode == M_LAYERS_DYNAMIC) {  // calibrate_minmax on this call's activations only
            const cudaError_t me = cudaMemsetAsync(s.act_amax, 0, sizeof(uint32_t) * 4 * s.layers, s.st);
            if (me != cudaSuccess) rc = cuda_fail(me, "cudaMemsetAsync (amax)");
        }
        if (!rc) rc = enqueue_layers(s, mode == M_LAYERS_DYNAMIC);
    }
    s.capturing = false;
    cudaError_t e = cudaStreamEndCapture(s.st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    {  // kernel launches per forward: the graph's kernel nodes
        size_t n = 0;
        if (cudaGraphGetNodes(g, nullptr, &n) == cudaSuccess && n) {
            std::vector<cudaGraphNode_t> nodes(n);
            if (cudaGraphGetNodes(g, nodes.data(), &n) == cudaSuccess) {
                int64_t k = 0;
                for (size_t i = 0; i < n; i++) {
                    cudaGraphNodeType t;
                    if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
                }
                s.graph_kernels[mode] = k;
            }
        }
    }
    e = cudaGraphInstantiate(&s.gexec[mode], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    return TVQ_OK;
}

// Queue one forward whose logits go to host memory, with every copy on the
// session's copy stream: the ids copy and the body on st, then the LM head
// (in row chunks when there are enough rows, each chunk's copy overlapping
// the next chunk), and copies_done recorded after the last copy.  Before
// the LM head overwrites a range of the device logits, st waits until the
// previous call's copy of that range is done, so calls can be queued back
// to back (the next forward's body runs while this one's logits cross PCIe).
int enqueue_host_logits(Session& s, const int64_t* ids, int ids_on_device, float* logits, cudaStream_t st) {
    const int chunk_rows = logit_chunk_rows();
    const bool chunked = s.logits_mode == 0 && chunk_rows > 0 && s.T >= 2 * chunk_rows && !s.profile;
    const int nch = chunked ? (s.T + chunk_rows - 1) / chunk_rows : 1;
    if (chunked && !s.gexec[M_BODY]) STEP(capture(s, M_BODY));
    if (!chunked && !s.gexec[M_FORWARD]) STEP(capture(s, M_FORWARD));
    if (!s.cp) TVQ_CUDA(cudaStreamCreateWithFlags(&s.cp, cudaStreamNonBlocking));
    if (!s.copies_done) TVQ_CUDA(cudaEventCreateWithFlags(&s.copies_done, cudaEventDisableTiming));
    while (static_cast<int>(s.chunk_ev.size()) < nch) {
        cudaEvent_t e = nullptr, f = nullptr;
        TVQ_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        s.chunk_ev.push_back(e);
        TVQ_CUDA(cudaEventCreateWithFlags(&f, cudaEventDisableTiming));
        s.copied_ev.push_back(f);
    }
    if (ids)
        TVQ_CUDA(cudaMemcpyAsync(s.ids, ids, sizeof(int64_t) * s.T,
                                 ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
    const int rows_all = static_cast<int>(s.logits_rows());
    if (!chunked) {
        // the LM head is inside the captured forward: it may not start
        // before the previous call's copy has read the device logits
        TVQ_CUDA(cudaStreamWaitEvent(st, s.copied_ev[0], 0));
        TVQ_CUDA(cudaGraphLaunch(s.gexec[M_FORWARD], st));
    } else {
        TVQ_CUDA(cudaGraphLaunch(s.gexec[M_BODY], st));
    }
    for (int c = 0; c < nch; c++) {
        const int r0 = chunked ? c * chunk_rows : 0;
        const int rows = chunked ? std::min(s.T - r0, chunk_rows) : rows_all;
        if (chunked) {
            TVQ_CUDA(cudaStreamWaitEvent(st, s.copied_ev[c], 0));  // no-op before the first copy
            STEP(launch_lm_head(s, r0, rows, st));
        }
        TVQ_CUDA(cudaEventRecord(s.chunk_ev[c], st));
        TVQ_CUDA(cudaStreamWaitEvent(s.cp, s.chunk_ev[c], 0));
        const size_t off = static_cast<size_t>(r0) * s.vocab;
        TVQ_CUDA(cudaMemcpyAsync(logits + off, s.logits + off, static_cast<size_t>(rows) * s.vocab * sizeof(float),
                                 cudaMemcpyDeviceToHost, s.cp));
        TVQ_CUDA(cudaEventRecord(s.copied_ev[c], s.cp));
    }
    TVQ_CUDA(cudaEventRecord(s.copies_done, s.cp));
    s.last_mode = chunked ? M_BODY : M_FORWARD;
    s.extra_launches = chunked ? nch : 0;
    return TVQ_OK;
}

}  // namespace
}  // namespace tvq

using namespace tvq;

extern "C" {

int tvq_session_create(int device, int64_t vocab, int64_t d_model, int64_t n_heads, int64_t n_layers, int64_t d_ffn,
                       int64_t max_pos, double ln_eps, int64_t max_tokens, int64_t* handle) {
    TVQ_CHECK(handle, TVQ_ERR_INVALID, "null handle pointer");
    TVQ_CHECK(vocab >= 0 && d_model > 0 && n_heads > 0 && n_layers >= 0 && d_ffn > 0 && max_pos > 0 && max_tokens > 0,
              TVQ_ERR_INVALID, "model sizes must be positive (vocab 0: a layer stack without embeddings)");
    TVQ_CHECK(d_model % n_heads == 0, TVQ_ERR_INVALID, "d_model must be a multiple of n_heads");
    TVQ_CHECK(d_model % 16 == 0 && d_ffn % 16 == 0, TVQ_ERR_UNSUPPORTED, "d_model and d_ffn must be multiples of 16");
    TVQ_CHECK(max_tokens < (1 << 30) && vocab < (1 << 30), TVQ_ERR_UNSUPPORTED, "size too large");
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    TVQ_CHECK(device >= 0 && device < ndev, TVQ_ERR_INVALID, "bad device ordinal");
    try {
        auto s = std::make_unique<Session>();
        s->device = device;
        DeviceGuard dg(device);
        if (dg.rc) return dg.rc;
        int rc = 0;
        DeviceState* ds = device_state(&rc);
        if (!ds) return rc;
        TVQ_CHECK(ds->cc_major == 10, TVQ_ERR_UNSUPPORTED, "sessions need an sm_100 device");
        s->vocab = static_cast<int>(vocab);
        s->d = static_cast<int>(d_model);
        s->heads = static_cast<int>(n_heads);
        s->layers = static_cast<int>(n_layers);
        s->ffn = static_cast<int>(d_ffn);
        s->max_pos = static_cast<int>(max_pos);
        s->max_tokens = static_cast<int>(max_tokens);
        s->eps = ln_eps;
        s->L.resize(static_cast<size_t>(n_layers));
        TVQ_CUDA(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
        const size_t MT = static_cast<size_t>(max_tokens), D = static_cast<size_t>(d_model);
        const size_t F = static_cast<size_t>(d_ffn);
        STEP(s->alloc(&s->act_scale, static_cast<size_t>(4 * std::max<int64_t>(n_layers, 1))));
        STEP(s->alloc(&s->act_amax, static_cast<size_t>(4 * std::max<int64_t>(n_layers, 1))));
        TVQ_CUDA(cudaMemset(s->act_amax, 0, sizeof(uint32_t) * 4 * std::max<int64_t>(n_layers, 1)));
        TVQ_CUDA(cudaMemset(s->act_scale, 0, sizeof(float) * 4 * std::max<int64_t>(n_layers, 1)));
        STEP(s->alloc(&s->ids, MT));
        STEP(s->alloc(&s->seg, MT + 1));
        STEP(s->alloc(&s->tok_start, MT));
        STEP(s->alloc(&s->x, MT * D));
        STEP(s->alloc(&s->qkv, MT * 3 * D));
        STEP(s->alloc(&s->hf, MT * std::max(D, F)));
        STEP(s->alloc(&s->xf, MT * D));
        STEP(s->alloc(&s->xf_last, MT * D));
        STEP(s->alloc(&s->xf_hi, MT * D));
        STEP(s->alloc(&s->xf_lo, MT * D));
        STEP(s->alloc(&s->xf_rs, MT));
        STEP(s->alloc(&s->aq, MT * D));
        STEP(s->alloc(&s->hq, MT * F));
        STEP(s->alloc(&s->err, 1));
        STEP(s->alloc(&s->kv_exp, static_cast<size_t>(3 * n_heads)));
        // head maxima of V per layer, then the fix-up lists' three counters
        STEP(s->alloc(&s->vmax, static_cast<size_t>(std::max<int64_t>(n_layers, 1) * d_model + 4)));
        s->fix_n = reinterpret_cast<int*>(s->vmax + std::max<int64_t>(n_layers, 1) * d_model);
        TVQ_CUDA(cudaMemset(s->vmax, 0, sizeof(uint32_t) * (std::max<int64_t>(n_layers, 1) * d_model + 4)));
        // (token, head) rows of one attention launch with undecided int8
        // columns: about 2 % at GPT-2 scales; room for 12.5 %
        s->fix_cap = static_cast<int>(std::min<int64_t>(std::max<int64_t>(4096, max_tokens * n_heads / 8), INT32_MAX / 16));
        STEP(s->alloc(&s->fix_list, static_cast<size_t>(s->fix_cap)));
        STEP(s->alloc(&s->fix_mask, static_cast<size_t>(s->fix_cap)));
        TVQ_CUDA(cudaMemset(s->err, 0, sizeof(int)));
        std::lock_guard<std::mutex> lk(g_mu);
        *handle = g_next++;
        g_sessions[*handle] = std::move(s);
        return TVQ_OK;
    } catch (const std::bad_alloc&) {
        set_error(TVQ_ERR_CUDA, "host allocation failed");
        return TVQ_ERR_CUDA;
    }
}

int tvq_session_destroy(int64_t handle) {
    std::unique_ptr<Session> s;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_sessions.find(handle);
        TVQ_CHECK(it != g_sessions.end(), TVQ_ERR_HANDLE, "unknown or destroyed session handle");
        s = std::move(it->second);
        g_sessions.erase(it);
    }
    DeviceGuard dg(s->device);
    cudaStreamSynchronize(s->st);
    s.reset();
    return TVQ_OK;
}

int tvq_session_set_embeddings(int64_t handle, const float* wte, const float* wpe) {
    SESSION(handle)
    TVQ_CHECK(wte && wpe, TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(S->vocab > 0, TVQ_ERR_INVALID, "the session was created without a vocabulary (layer stack)");
    const size_t vd = static_cast<size_t>(S->vocab) * S->d;
    if (!S->wte) STEP(S->alloc(&S->wte, vd));
    if (!S->wte_hi) STEP(S->alloc(&S->wte_hi, vd));
    if (!S->wte_lo) STEP(S->alloc(&S->wte_lo, vd));
    if (!S->wte_rs) STEP(S->alloc(&S->wte_rs, static_cast<size_t>(S->vocab)));
    if (!S->wpe) STEP(S->alloc(&S->wpe, static_cast<size_t>(S->max_pos) * S->d));
    TVQ_CUDA(cudaMemcpy(S->wte, wte, sizeof(float) * vd, cudaMemcpyHostToDevice));
    TVQ_CUDA(cudaMemcpy(S->wpe, wpe, sizeof(float) * S->max_pos * S->d, cudaMemcpyHostToDevice));
    STEP(launch_split_f16_rows(S->wte, S->wte_hi, S->wte_lo, S->wte_rs, S->vocab, S->d, S->st));
    TVQ_CUDA(cudaStreamSynchronize(S->st));
    return TVQ_OK;
}

int tvq_session_set_layernorm(int64_t handle, int64_t layer, int64_t which, const float* gamma, const float* beta) {
    SESSION(handle)
    TVQ_CHECK(gamma && beta, TVQ_ERR_INVALID, "null buffer");
    TVQ_CHECK(layer >= -1 && layer < S->layers, TVQ_ERR_INVALID, "bad layer");
    float **g, **b;
    if (layer < 0) {
        g = &S->lnf_g;
        b = &S->lnf_b;
    } else {
        TVQ_CHECK(which == 0 || which == 1, TVQ_ERR_INVALID, "which must be 0 (ln_1) or 1 (ln_2)");
        g = &S->L[layer].ln[2 * which];
        b = &S->L[layer].ln[2 * which + 1];
    }
    if (!*g) STEP(S->alloc(g, S->d));
    if (!*b) STEP(S->alloc(b, S->d));
    TVQ_CUDA(cudaMemcpy(*g, gamma, sizeof(float) * S->d, cudaMemcpyHostToDevice));
    TVQ_CUDA(cudaMemcpy(*b, beta, sizeof(float) * S->d, cudaMemcpyHostToDevice));
    return TVQ_OK;
}

// After a linear's int8 weights, scales and bias are in place: the per-head
// K / V bounds of a c_attn layer with head dim 64 (for the epilogue's split).
static int lin_finish(Session* S, Lin& l, int64_t which) {
    if (which == 0 && S->heads > 0 && S->d == 64 * S->heads) {
        if (!l.kvb) STEP(S->alloc(&l.kvb, static_cast<size_t>(6 * S->heads)));
        STEP(launch_kv_head_bound(l.W, l.sw, l.bias, l.k, S->d, l.kvb, S->st));
        TVQ_CUDA(cudaStreamSynchronize(S->st));
    }
    l.set = true;
    return check_device_error(S->st);
}

static int lin_alloc(Session* S, Lin& l, int n, int k) {
    if (!l.W) {
        STEP(S->alloc(&l.W, static_cast<size_t>(n) * k));
        STEP(S->alloc(&l.sw, static_cast<size_t>(n)));
        STEP(S->alloc(&l.bias, static_cast<size_t>(n)));
    }
    l.n = n;
    l.k = k;
    return TVQ_OK;
}

int tvq_session_set_linear_f32(int64_t handle, int64_t layer, int64_t which, const float* w, const float* bias,
                               int layout) {
    SESSION(handle)
    TVQ_CHECK(layer >= 0 && layer < S->layers && which >= 0 && which < 4, TVQ_ERR_INVALID, "bad layer/which");
    TVQ_CHECK(w && bias && (layout == 0 || layout == 1), TVQ_ERR_INVALID, "bad arguments");
    int n, k;
    lin_shape(*S, static_cast<int>(which), &n, &k);
    Lin& l = S->L[layer].lin[which];
    STEP(lin_alloc(S, l, n, k));
    float *tmp = nullptr, *tmp2 = nullptr;
    const size_t nk = static_cast<size_t>(n) * k;
    TVQ_CUDA(cudaMalloc(&tmp, nk * sizeof(float) * 2));
    tmp2 = tmp + nk;
    int rc = TVQ_OK;
    cudaError_t e = cudaMemcpyAsync(tmp, w, nk * sizeof(float), cudaMemcpyHostToDevice, S->st);
    if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpy weights");
    const float* src = tmp;
    if (!rc && layout == 0) {  // HF Conv1D / gpt2_ref layout w[k * n + o]
        rc = launch_transpose(tmp, tmp2, k, n, S->st);
        src = tmp2;
    }
    // per-output-channel calibrate + quantize (engine.tkv:202-213, 237-250)
    if (!rc) rc = launch_rowwise(0, src, l.W, l.sw, n, k, S->st);
    if (!rc) {
        e = cudaMemcpyAsync(l.bias, bias, n * sizeof(float), cudaMemcpyHostToDevice, S->st);
        if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpy bias");
    }
    cudaStreamSynchronize(S->st);
    cudaFree(tmp);
    if (rc) return rc;
    return lin_finish(S, l, which);
}

int tvq_session_set_linear_i8(int64_t handle, int64_t layer, int64_t which, const int8_t* w_nk, const float* scales_w,
                              const float* bias) {
    SESSION(handle)
    TVQ_CHECK(layer >= 0 && layer < S->layers && which >= 0 && which < 4, TVQ_ERR_INVALID, "bad layer/which");
    TVQ_CHECK(w_nk && scales_w && bias, TVQ_ERR_INVALID, "null buffer");
    int n, k;
    lin_shape(*S, static_cast<int>(which), &n, &k);
    Lin& l = S->L[layer].lin[which];
    STEP(lin_alloc(S, l, n, k));
    TVQ_CUDA(cudaMemcpy(l.W, w_nk, static_cast<size_t>(n) * k, cudaMemcpyHostToDevice));
    TVQ_CUDA(cudaMemcpy(l.sw, scales_w, sizeof(float) * n, cudaMemcpyHostToDevice));
    TVQ_CUDA(cudaMemcpy(l.bias, bias, sizeof(float) * n, cudaMemcpyHostToDevice));
    return lin_finish(S, l, which);
}

int tvq_session_get_linear_i8(int64_t handle, int64_t layer, int64_t which, int8_t* w_nk, float* scales_w) {
    SESSION(handle)
    TVQ_CHECK(layer >= 0 && layer < S->layers && which >= 0 && which < 4, TVQ_ERR_INVALID, "bad layer/which");
    Lin& l = S->L[layer].lin[which];
    TVQ_CHECK(l.set, TVQ_ERR_INVALID, "linear not set");
    if (w_nk) TVQ_CUDA(cudaMemcpy(w_nk, l.W, static_cast<size_t>(l.n) * l.k, cudaMemcpyDeviceToHost));
    if (scales_w) TVQ_CUDA(cudaMemcpy(scales_w, l.sw, sizeof(float) * l.n, cudaMemcpyDeviceToHost));
    return TVQ_OK;
}

int tvq_session_set_act_scales(int64_t handle, const float* scales, int64_t n) {
    SESSION(handle)
    TVQ_CHECK(scales && n == 4LL * S->layers, TVQ_ERR_SIZE, "need 4 scales per layer");
    if (n) TVQ_CUDA(cudaMemcpy(S->act_scale, scales, sizeof(float) * n, cudaMemcpyHostToDevice));
    return TVQ_OK;
}

int tvq_session_get_act_scales(int64_t handle, float* scales, int64_t n) {
    SESSION(handle)
    TVQ_CHECK(scales && n >= 4LL * S->layers, TVQ_ERR_SIZE, "need room for 4 scales per layer");
    TVQ_CUDA(cudaStreamSynchronize(S->st));
    if (S->layers) TVQ_CUDA(cudaMemcpy(scales, S->act_scale, sizeof(float) * 4 * S->layers, cudaMemcpyDeviceToHost));
    return TVQ_OK;
}

int tvq_session_prepare(int64_t handle, const int64_t* seg, int64_t n_seg, int logits_mode) {
    SESSION(handle)
    TVQ_CHECK(seg && n_seg >= 1, TVQ_ERR_INVALID, "need at least one sequence");
    TVQ_CHECK(logits_mode == 0 || logits_mode == 1, TVQ_ERR_INVALID, "logits_mode must be 0 (all) or 1 (last)");
    TVQ_CHECK(seg[0] == 0, TVQ_ERR_INVALID, "seg[0] must be 0");
    const int64_t T = seg[n_seg];
    TVQ_CHECK(T >= 1 && T <= S->max_tokens, TVQ_ERR_SIZE, "token count exceeds the session's max_tokens");
    std::vector<int> sh(static_cast<size_t>(n_seg) + 1);
    std::vector<int> tok(static_cast<size_t>(T));
    // attention work: one item per query tile (128 rows on the tensor-core
    // path, else 64), or, when its causal key range is longer than kKeyChunk,
    // one item per key chunk plus a merge.  Chunks start at multiples of
    // kKeyChunk (a multiple of the tile height) from the sequence start, so
    // every row of a tile sees at least one key of every chunk.
    // TVQ_ATTN_TC=0 selects the fp32 kernel; TVQ_ATTN_KEY_CHUNK overrides the
    // chunk (keys, rounded to the tile height; 0 = never split).
    const bool tc = S->heads > 0 && S->d / S->heads == 64 && !(getenv("TVQ_ATTN_TC") && atoi(getenv("TVQ_ATTN_TC")) == 0);
    const int QT = tc ? attention_tc_rows() : 64;
    // Key chunks exist to give the SMs enough units when a few long
    // sequences make few query tiles (one 1024-token sequence: 8 tiles x 12
    // heads for 148 SMs).  A layout with at least 8 unsplit units per SM (a
    // packed batch of requests) keeps whole tiles: its splits only add partial
    // merges (measured: config 4's attention 24.9 -> 21.3 ms per step, config
    // 5's 11.2 -> 8.1 ms without them; config 2 is faster with them).
    int kKeyChunk = 512;
    {
        int64_t qtiles = 0;
        for (int64_t s = 0; s < n_seg; s++)
            if (seg[s + 1] > seg[s]) qtiles += (seg[s + 1] - seg[s] + QT - 1) / QT;
        int rc2 = 0;
        DeviceState* ds = device_state(&rc2);
        const int sms = ds ? ds->sm_count : 148;
        if (qtiles * S->heads >= 8LL * sms) kKeyChunk = 1 << 30;
    }
    if (const char* env = getenv("TVQ_ATTN_KEY_CHUNK")) {
        const int v = atoi(env);
        kKeyChunk = v <= 0 ? (1 << 30) : std::max(QT, v / QT * QT);
    }
    struct Item { int4 tile, split; int work; };
    std::vector<Item> items;
    std::vector<int4> comb;
    int nparts = 0;
    for (int64_t s = 0; s < n_seg; s++) {
        const int64_t a = seg[s], b = seg[s + 1];
        TVQ_CHECK(b > a, TVQ_ERR_INVALID, "every sequence needs at least one token");
        TVQ_CHECK(b - a <= S->max_pos, TVQ_ERR_SIZE, "sequence longer than max_pos");
        for (int64_t t = a; t < b; t++) tok[t] = static_cast<int>(a);
        for (int64_t q0 = a; q0 < b; q0 += QT) {
            const int kend = static_cast<int>(std::min<int64_t>(q0 + QT, b));
            const int len = kend - static_cast<int>(a);
            const int4 tile = make_int4(static_cast<int>(q0), static_cast<int>(a), static_cast<int>(b), 0);
            if (len <= kKeyChunk) {
                items.push_back({tile, make_int4(static_cast<int>(a), kend, -1, 0), len});
            } else {
                const int first = nparts;
                int nch = 0;
                for (int kb = static_cast<int>(a); kb < kend; kb += kKeyChunk, nch++)
                    items.push_back({tile, make_int4(kb, std::min(kb + kKeyChunk, kend), nparts++,
                                                     static_cast<int>(comb.size())),
                                     std::min(kKeyChunk, kend - kb)});
                comb.push_back(make_int4(static_cast<int>(q0), static_cast<int>(b), first, nch));
            }
        }
        sh[s] = static_cast<int>(a);
    }
    sh[n_seg] = static_cast<int>(T);
    // longest causal work first (grouping each sequence's items together,
    // for its K / V blocks to be shared in L2, measured slower: config 4
    // attention 24.1 -> 25.3 ms per step; the balance across CTAs matters more)
    std::stable_sort(items.begin(), items.end(), [](const Item& u, const Item& v) { return u.work > v.work; });
    std::vector<int4> tiles(items.size()), splits(items.size());
    for (size_t i = 0; i < items.size(); i++) {
        tiles[i] = items[i].tile;
        splits[i] = items[i].split;
    }
    TVQ_CUDA(cudaStreamSynchronize(S->st));
    auto grow = [&](auto** ptr, size_t& cap, size_t want) -> int {
        if (want <= cap) return TVQ_OK;
        if (*ptr) {
            cudaFree(*ptr);
            S->allocs.erase(std::remove(S->allocs.begin(), S->allocs.end(), static_cast<void*>(*ptr)), S->allocs.end());
            *ptr = nullptr;
        }
        int r = S->alloc(ptr, want);
        if (!r) cap = want;
        return r;
    };
    STEP(grow(&S->tiles, S->tiles_cap, items.size()));
    STEP(grow(&S->split, S->split_cap, items.size()));
    STEP(grow(&S->comb, S->comb_cap, std::max<size_t>(comb.size(), 1)));
    const size_t slots = static_cast<size_t>(std::max(nparts, 1)) * S->heads * QT;
    STEP(grow(&S->part_o, S->part_o_cap, slots * (S->d / S->heads)));
    STEP(grow(&S->part_ml, S->part_ml_cap, slots));
    STEP(grow(&S->counters, S->counters_cap, std::max<size_t>(comb.size(), 1) * S->heads));
    TVQ_CUDA(cudaMemset(S->counters, 0, sizeof(int) * std::max<size_t>(comb.size(), 1) * S->heads));
    TVQ_CUDA(cudaMemcpy(S->seg, sh.data(), sizeof(int) * sh.size(), cudaMemcpyHostToDevice));
    TVQ_CUDA(cudaMemcpy(S->tok_start, tok.data(), sizeof(int) * tok.size(), cudaMemcpyHostToDevice));
    TVQ_CUDA(cudaMemcpy(S->tiles, tiles.data(), sizeof(int4) * tiles.size(), cudaMemcpyHostToDevice));
    TVQ_CUDA(cudaMemcpy(S->split, splits.data(), sizeof(int4) * splits.size(), cudaMemcpyHostToDevice));
    if (!comb.empty()) TVQ_CUDA(cudaMemcpy(S->comb, comb.data(), sizeof(int4) * comb.size(), cudaMemcpyHostToDevice));
    S->ncomb = static_cast<int>(comb.size());
    S->attn_tc = tc;
    S->attn_rows = QT;
    if (tc && !S->kh) {
        const size_t n = static_cast<size_t>(attention_tc_pitch(S->max_tokens)) * S->d;
        STEP(S->alloc(&S->qh, n));
        STEP(S->alloc(&S->ql, n));
        STEP(S->alloc(&S->kh, n));
        STEP(S->alloc(&S->kl, n));
        STEP(S->alloc(&S->vh, n));
        STEP(S->alloc(&S->vl, n));
    }
    S->T = static_cast<int>(T);
    S->nseg = static_cast<int>(n_seg);
    S->ntiles = static_cast<int>(tiles.size());
    S->logits_mode = logits_mode;
    S->seg_host = sh;
    const size_t need = static_cast<size_t>(S->logits_rows()) * S->vocab;
    if (need > S->logits_cap) {
        if (S->logits) {
            cudaFree(S->logits);
            S->allocs.erase(std::remove(S->allocs.begin(), S->allocs.end(), static_cast<void*>(S->logits)),
                            S->allocs.end());
            S->logits = nullptr;
        }
        STEP(S->alloc(&S->logits, need));
        S->logits_cap = need;
    }
    S->prepared = true;
    S->drop_graphs();
    return TVQ_OK;
}

int tvq_session_calibrate(int64_t handle, const int64_t* ids, int ids_on_device, int reset) {
    SESSION(handle)
    STEP(check_ready(*S));
    TVQ_CHECK(ids, TVQ_ERR_INVALID, "null ids");
    // a queued tvq_session_forward_async's copies still read the device logits
    if (S->copies_done) TVQ_CUDA(cudaStreamWaitEvent(S->st, S->copies_done, 0));
    if (reset && S->layers)
        TVQ_CUDA(cudaMemsetAsync(S->act_amax, 0, sizeof(uint32_t) * 4 * S->layers, S->st));
    TVQ_CUDA(cudaMemcpyAsync(S->ids, ids, sizeof(int64_t) * S->T,
                             ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, S->st));
    STEP(enqueue_forward(*S, true));
    return check_err(*S, S->st);
}

int tvq_session_forward(int64_t handle, const int64_t* ids, int ids_on_device, float* logits, int64_t logits_len,
                        int logits_on_device, void* stream) {
    SESSION(handle)
    STEP(check_ready(*S));
    const size_t out_elems = static_cast<size_t>(S->logits_rows()) * S->vocab;
    TVQ_CHECK(!logits || logits_len >= static_cast<int64_t>(out_elems), TVQ_ERR_SIZE, "logits buffer too small");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : S->st;
    const int chunk_rows = logit_chunk_rows();
    if (logits && !logits_on_device && S->logits_mode == 0 && chunk_rows > 0 && S->T >= 2 * chunk_rows &&
        !S->profile) {
        // all logits to the host: the LM head runs in row chunks after the
        // captured body, and each chunk's rows are copied out on a second
        // stream while the next chunk computes (the copy, not the GEMM,
        // bounds this call)
        STEP(enqueue_host_logits(*S, ids, ids_on_device, logits, st));
        TVQ_CUDA(cudaStreamWaitEvent(st, S->copies_done, 0));
        return check_err(*S, st);
    }
    if (!S->gexec[M_FORWARD]) STEP(capture(*S, M_FORWARD));
    if (S->copies_done) TVQ_CUDA(cudaStreamWaitEvent(st, S->copies_done, 0));  // a queued call's copies read the logits
    if (ids)
        TVQ_CUDA(cudaMemcpyAsync(S->ids, ids, sizeof(int64_t) * S->T,
                                 ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
    TVQ_CUDA(cudaGraphLaunch(S->gexec[M_FORWARD], st));
    S->last_mode = M_FORWARD;
    S->extra_launches = 0;
    if (logits)
        TVQ_CUDA(cudaMemcpyAsync(logits, S->logits, out_elems * sizeof(float),
                                 logits_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
    if ((ids && !ids_on_device) || (logits && !logits_on_device)) return check_err(*S, st);
    return TVQ_OK;
}

int tvq_session_forward_async(int64_t handle, const int64_t* ids, int ids_on_device, float* logits, int64_t logits_len,
                              void* stream) {
    SESSION(handle)
    STEP(check_ready(*S));
    TVQ_CHECK(logits, TVQ_ERR_INVALID, "a host logits buffer is required");
    const size_t out_elems = static_cast<size_t>(S->logits_rows()) * S->vocab;
    TVQ_CHECK(logits_len >= static_cast<int64_t>(out_elems), TVQ_ERR_SIZE, "logits buffer too small");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : S->st;
    return enqueue_host_logits(*S, ids, ids_on_device, logits, st);
}

int tvq_session_join(int64_t handle, void* stream) {
    SESSION(handle)
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : S->st;
    if (S->copies_done) TVQ_CUDA(cudaStreamWaitEvent(st, S->copies_done, 0));
    return TVQ_OK;
}

int tvq_session_wait(int64_t handle, void* stream) {
    SESSION(handle)
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : S->st;
    if (S->copies_done) TVQ_CUDA(cudaStreamWaitEvent(st, S->copies_done, 0));
    return check_err(*S, st);
}

int tvq_session_run_layers(int64_t handle, const float* x, int x_on_device, float* y, int y_on_device, int dynamic,
                           void* stream) {
    SESSION(handle)
    STEP(check_ready(*S, true));
    TVQ_CHECK(dynamic == 0 || dynamic == 1, TVQ_ERR_INVALID, "dynamic must be 0 (static scales) or 1");
    const int mode = dynamic ? M_LAYERS_DYNAMIC : M_LAYERS;
    if (!S->gexec[mode]) STEP(capture(*S, mode));
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : S->st;
    const size_t bytes = sizeof(float) * static_cast<size_t>(S->T) * S->d;
    if (x) TVQ_CUDA(cudaMemcpyAsync(S->x, x, bytes, x_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
    TVQ_CUDA(cudaGraphLaunch(S->gexec[mode], st));
    S->last_mode = mode;
    S->extra_launches = 0;
    if (y) TVQ_CUDA(cudaMemcpyAsync(y, S->x, bytes, y_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
    if ((x && !x_on_device) || (y && !y_on_device)) return check_err(*S, st);
    return TVQ_OK;
}

int tvq_session_hidden(int64_t handle, float** x_dev) {
    SESSION(handle)
    TVQ_CHECK(x_dev, TVQ_ERR_INVALID, "null out pointer");
    *x_dev = S->x;
    return TVQ_OK;
}

int tvq_session_logits(int64_t handle, float** logits_dev, int64_t* rows, int64_t* cols) {
    SESSION(handle)
    TVQ_CHECK(logits_dev, TVQ_ERR_INVALID, "null out pointer");
    *logits_dev = S->logits;
    if (rows) *rows = S->prepared ? S->logits_rows() : 0;
    if (cols) *cols = S->vocab;
    return TVQ_OK;
}

int tvq_session_set_profiling(int64_t handle, int enable) {
    SESSION(handle)
    S->profile = enable != 0;
    S->drop_graphs();  // recapture with or without the stage events
    return TVQ_OK;
}

int tvq_session_stage_times(int64_t handle, float* ms, int64_t n) {
    SESSION(handle)
    TVQ_CHECK(ms && n >= ST_COUNT, TVQ_ERR_SIZE, "need room for every stage");
    TVQ_CHECK(S->profile && S->ev.size() >= 2, TVQ_ERR_INVALID, "profiling is off or no forward has run");
    for (int i = 0; i < ST_COUNT; i++) ms[i] = 0.0f;
    TVQ_CUDA(cudaEventSynchronize(S->ev.back()));
    for (size_t i = 1; i < S->ev.size(); i++) {
        float t = 0.0f;
        TVQ_CUDA(cudaEventElapsedTime(&t, S->ev[i - 1], S->ev[i]));
        if (S->ev_stage[i] >= 0) ms[S->ev_stage[i]] += t;
    }
    return TVQ_OK;
}

int tvq_session_launches(int64_t handle, int64_t* kernels) {
    SESSION(handle)
    TVQ_CHECK(kernels, TVQ_ERR_INVALID, "null output pointer");
    TVQ_CHECK(S->last_mode >= 0 && S->gexec[S->last_mode], TVQ_ERR_INVALID,
              "no forward has been captured for this layout");
    *kernels = S->graph_kernels[S->last_mode] + S->extra_launches;
    return TVQ_OK;
}

int tvq_session_sync(int64_t handle) {
    SESSION(handle)
    return check_err(*S, S->st);
}

// ---------------------------------------------------------------- glue kernels, device buffers

int tvq_dev_layernorm(const float* x, const float* gamma, const float* beta, float* y, int8_t* q,
                      const float* qscale_dev, uint32_t* amax_dev, int64_t rows, int64_t d, double eps,
                      void* stream) {
    TVQ_CHECK(rows >= 0 && d > 0 && x && gamma && beta && (y || q || amax_dev), TVQ_ERR_INVALID, "bad arguments");
    TVQ_CHECK(!q || qscale_dev, TVQ_ERR_INVALID, "int8 output needs a scale");
    return launch_layernorm(x, gamma, beta, y, q, qscale_dev, amax_dev, static_cast<int>(rows), static_cast<int>(d),
                            eps, static_cast<cudaStream_t>(stream));
}

int tvq_dev_attention(const float* qkv, const int64_t* seg, int64_t n_seg, int64_t d, int64_t n_heads,
                      int32_t* tiles_dev32, int64_t tiles_cap, float* out, int8_t* outq, const float* qscale_dev,
                      uint32_t* amax_dev, void* stream) {
    int4* tiles_dev = reinterpret_cast<int4*>(tiles_dev32);
    TVQ_CHECK((reinterpret_cast<uintptr_t>(tiles_dev32) & 15) == 0, TVQ_ERR_UNSUPPORTED, "tile buffer must be 16-byte aligned");
    TVQ_CHECK(qkv && seg && n_seg >= 1 && tiles_dev && (out || outq || amax_dev), TVQ_ERR_INVALID, "bad arguments");
    TVQ_CHECK(!outq || qscale_dev, TVQ_ERR_INVALID, "int8 output needs a scale");
    TVQ_CHECK(n_heads > 0 && d > 0 && n_heads <= d && d % n_heads == 0 && d < (1LL << 29), TVQ_ERR_INVALID,
              "d must be a positive multiple of the head count");
    TVQ_CHECK(seg[0] >= 0 && seg[n_seg] < (1LL << 31), TVQ_ERR_INVALID,
              "segment offsets must lie in [0, 2^31)");
    // head dim 64: the tensor-core kernel, 128-row query tiles with their key
    // ranges (two entries per tile); otherwise the fp32 kernel, 64-row tiles
    const bool tc = d / n_heads == 64;
    const int rows = tc ? attention_tc_rows() : 64;
    std::vector<int4> tiles, keys;
    for (int64_t s = 0; s < n_seg; s++) {
        TVQ_CHECK(seg[s + 1] >= seg[s], TVQ_ERR_INVALID, "segments must be non-decreasing");
        for (int64_t q0 = seg[s]; q0 < seg[s + 1]; q0 += rows) {
            tiles.push_back(make_int4(static_cast<int>(q0), static_cast<int>(seg[s]), static_cast<int>(seg[s + 1]), 0));
            keys.push_back(make_int4(static_cast<int>(seg[s]), static_cast<int>(std::min(q0 + rows, seg[s + 1])), -1, 0));
        }
    }
    const int64_t n = static_cast<int64_t>(tiles.size());
    TVQ_CHECK((tc ? 2 * n : n) <= tiles_cap, TVQ_ERR_SIZE, "tile buffer too small");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n) TVQ_CUDA(cudaMemcpyAsync(tiles_dev, tiles.data(), sizeof(int4) * n, cudaMemcpyHostToDevice, st));
    if (n && tc) TVQ_CUDA(cudaMemcpyAsync(tiles_dev + n, keys.data(), sizeof(int4) * n, cudaMemcpyHostToDevice, st));
    TVQ_CUDA(cudaStreamSynchronize(st));  // the host vectors die at return
    if (tc) {
        // split K / V scratch, stream-ordered (freed when the kernel is done)
        const int T = static_cast<int>(seg[n_seg]);
        // fp16 Q / K / V^T hi + lo (n4 halves each), then 3 heads exponents
        // and 3 heads amax words
        const size_t n4 = std::max<size_t>((static_cast<size_t>(attention_tc_pitch(T)) * d + 7) & ~size_t(7), 8);
        // + the exact-int8 fix-up list (16-byte rows, 8-byte column masks)
        // and three counters
        const int64_t fcap = outq ? std::max<int64_t>(4096, static_cast<int64_t>(T) * n_heads / 8) : 0;
        TVQ_CHECK(fcap <= INT32_MAX / 16, TVQ_ERR_UNSUPPORTED, "too many tokens x heads for the int8 fix-up lists");
        uint16_t* kv = nullptr;
        const size_t kv_bytes =
            (sizeof(uint16_t) * 6 * n4 + sizeof(int) * 6 * n_heads + 4 * sizeof(int) + sizeof(uint32_t) * d + 15) &
            ~size_t(15);
        TVQ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&kv),
                                 kv_bytes + (sizeof(int4) + sizeof(uint2)) * static_cast<size_t>(fcap), st));
        int* kv_exp = reinterpret_cast<int*>(kv + 6 * n4);
        uint32_t* kv_amax = reinterpret_cast<uint32_t*>(kv_exp + 3 * n_heads);
        AttnFix fx;
        fx.n = reinterpret_cast<int*>(kv_amax + 3 * n_heads);
        uint32_t* vcol = reinterpret_cast<uint32_t*>(fx.n + 4);  // each V column's max |V| (launch_split_kv)
        fx.vmax = vcol;
        fx.list = reinterpret_cast<int4*>(reinterpret_cast<char*>(kv) + kv_bytes);
        fx.mask = reinterpret_cast<uint2*>(fx.list + fcap);
        fx.cap = static_cast<int>(fcap);
        if (fcap) TVQ_CUDA(cudaMemsetAsync(fx.n, 0, 3 * sizeof(int), st));
        int r = launch_split_kv(qkv, T, static_cast<int>(d), kv, kv + n4, kv + 2 * n4, kv + 3 * n4, kv + 4 * n4,
                                kv + 5 * n4, kv_exp, kv_amax, st, fcap ? vcol : nullptr);
        if (!r)
            r = launch_attention_tc(qkv, kv, kv + n4, kv + 2 * n4, kv + 3 * n4, kv + 4 * n4, kv + 5 * n4, kv_exp, T,
                                    tiles_dev, tiles_dev + n,
                                    static_cast<int>(n), nullptr, 0, static_cast<int>(d), static_cast<int>(n_heads), out,
                                    outq, qscale_dev, amax_dev, nullptr, nullptr, nullptr, st, fcap ? &fx : nullptr);
        cudaError_t e = cudaFreeAsync(kv, st);
        if (!r && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
        return r;
    }
    return launch_attention(qkv, tiles_dev, static_cast<int>(n), static_cast<int>(seg[n_seg]), static_cast<int>(d),
                            static_cast<int>(n_heads), out, outq, qscale_dev, amax_dev, st);
}

}  // extern "C"
