// tvq_glue.h -- launchers of the fp32 GPT-2 glue kernels (tvq_glue.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tvq {

int launch_embed(const int64_t* ids, const int* tok_seg_start, const float* wte, const float* wpe, float* x, int T,
                 int d, int vocab, int max_pos, int* err, cudaStream_t st);
// y (f32) and/or q (int8 with qscale) and/or amax of y
// LayerNorm with its output as the row-scaled fp16 split of the LM head
// (launch_split_f16_rows's hi / lo [T, d] and rscale [T]); block per row.
int launch_layernorm_split(const float* x, const float* g, const float* b, void* hi, void* lo, float* rscale, int T,
                           int d, double eps, cudaStream_t st);
int launch_layernorm(const float* x, const float* g, const float* b, float* y, int8_t* q, const float* qscale,
                     uint32_t* amax, int T, int d, double eps, cudaStream_t st);
// tiles: int4 {q0, seg_start, seg_end, 0} per 64-row query tile
int launch_attention(const float* qkv, const int4* tiles, int ntiles, int T, int d, int nheads, float* out,
                     int8_t* outq, const float* qscale, uint32_t* amax, cudaStream_t st);
// split-KV form: split[i] = {key begin, key end, partial slot or -1, 0} per
// item; comb[e] = {q0, seq end, first partial slot, count} merges partials
// (part_o: slots x heads x 64 x hd floats, part_ml: slots x heads x 64).
int launch_attention_split(const float* qkv, const int4* tiles, const int4* split, int nitems, const int4* comb,
                           int ncomb, int d, int nheads, float* out, int8_t* outq, const float* qscale,
                           uint32_t* amax, float* part_o, float2* part_ml, cudaStream_t st);
int launch_attention_combine(const int4* comb, int ncomb, int d, int nheads, int rows, const float* part_o,
                             const float2* part_ml, float* out, int8_t* outq, const float* qscale, uint32_t* amax,
                             cudaStream_t st);
// tvq_attn_tc.cu: head dim 64 on the tensor cores.  The Q and K parts of
// qkv as fp16 hi / lo [T, d] and the V part transposed, V^T hi / lo [d,
// attention_tc_pitch(T)], head h of part p (0 Q, 1 K, 2 V) scaled by
// 2^kv_exp[p heads + h] so that its values stay below 2^15: written by the
// c_attn GEMM epilogue in a session, or by launch_split_kv (exact per-head
// max |.| into amax[3 heads], optionally each V column's max |V| into
// vcol[d], then the split).  launch_attention_tc takes
// them with the same work items as above but attention_tc_rows() (128) query
// rows per tile; split[] is required.
int attention_tc_rows();
int attention_tc_pitch(int T);
int launch_split_kv(const float* qkv, int T, int d, void* qh, void* ql, void* kh, void* kl, void* vth, void* vtl,
                    int* kv_exp, uint32_t* amax, cudaStream_t st, uint32_t* vcol = nullptr);
// Per-head bounds [6 d / 64] of a c_attn layer (W int8 [3d, k], per-channel
// sw, bias or null) for the epilogue's Q / K / V split (GemmArgs::kv_bound).
int launch_kv_head_bound(const int8_t* W, const float* sw, const float* bias, int k, int kvd, float* out,
                         cudaStream_t st);
// Exact int8 context (optional, with outq): vmax [d] = max |V| per V column
// (float bits); list [cap] rows whose int8 context has undecided columns
// {q, row max, head, sequence start}, mask [cap] those columns; n: three
// device ints (rows, rows taken, finished fix-up CTAs), zero before the first
// launch (the fix-up kernel leaves them zero).  The fix-up reads the f32
// qkv, so qkv must hold the values.  A launch with more undecided rows than
// cap records a device error (DEVERR_FIX_FULL).
struct AttnFix {
    const uint32_t* vmax = nullptr;
    int4* list = nullptr;
    uint2* mask = nullptr;
    int* n = nullptr;
    int cap = 0;
};
int launch_attention_tc(const float* qkv, const void* qh, const void* ql, const void* kh, const void* kl,
                        const void* vth, const void* vtl, const int* kv_exp, int T, const int4* tiles,
                        const int4* split, int nitems, const int4* comb, int ncomb, int d, int nheads, float* out,
                        int8_t* outq, const float* qscale, uint32_t* amax, float* part_o, float2* part_ml,
                        int* counters, cudaStream_t st, const AttnFix* fix = nullptr);
int launch_scale_from_amax(const uint32_t* amax, float* scale, int n, cudaStream_t st);
int launch_transpose(const float* a, float* b, int rows, int cols, cudaStream_t st);
int launch_token_seg(const int* seg, int nseg, int* tok_start, cudaStream_t st);
int launch_gather_last(const float* src, const int* seg, int nseg, int64_t n, float* dst, cudaStream_t st);

}  // namespace tvq
