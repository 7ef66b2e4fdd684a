/*
 * motif_b200 — C ABI of the B200 (sm_100a) kernels behind the Motif Chord inference path.
 *
 * Every entry point takes plain device pointers, sizes and element strides, launches on
 * the given CUDA stream (passed as `void*`, i.e. a `cudaStream_t`; NULL = legacy default
 * stream), never allocates, never synchronises, and returns an `MB_*` status code.  On a
 * nonzero code nothing was launched and `motif_b200_last_error()` holds a message.
 *
 * Dtype codes: MB_F32 / MB_F16 / MB_BF16 name the element type of the tensors marked
 * "dtype" in each signature; recurrent states, log-decays, write strengths, `log_n` and
 * the per-head GGD parameters are always fp32.
 *
 * Each declaration cites the reference interface it replaces (paths relative to the
 * reference project, CodonProject/codon-motif).  The Python shim `motif_b200/_lib.py`
 * binds these with ctypes and maps the codes onto the reference's exception types
 * (ValueError for MB_ERR_ARG/SHAPE/DTYPE/ALIGN, NotImplementedError for
 * MB_ERR_UNSUPPORTED, RuntimeError for MB_ERR_CUDA).
 */
#ifndef MOTIF_B200_H
#define MOTIF_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define MB_API __attribute__((visibility("default")))
#else
#define MB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MB_OK = 0,
  MB_ERR_ARG = 1,         /* null pointer or invalid scalar argument */
  MB_ERR_SHAPE = 2,       /* inconsistent sizes */
  MB_ERR_DTYPE = 3,       /* unsupported dtype code */
  MB_ERR_ALIGN = 4,       /* pointer / stride not aligned as required */
  MB_ERR_UNSUPPORTED = 5, /* valid call this build has no kernel for (e.g. head dim) */
  MB_ERR_CUDA = 6         /* the CUDA runtime reported an error at launch */
};

enum { MB_F32 = 0, MB_F16 = 1, MB_BF16 = 2 };

/* Message of the last failing call on this host thread ("" if none). */
MB_API const char* motif_b200_last_error(void);
/* ABI version of this library (bumped on any signature change). */
MB_API int motif_b200_abi_version(void);

/* ------------------------------------------------------------------ gated delta rule
 * Layout of `strides` (elements), [18]:
 *   q(b,h,l) k(b,h,l) v(b,h,l) o(b,h,l) beta(b,h,l) g(b,h,l)
 * q,k: [B,H,L,Dk] dtype, last dim contiguous; v,o: [B,H,L,Dv] dtype; beta,g: [B,H,L] fp32;
 * state_in / state_out: [B,H,Dk,Dv] fp32 contiguous; state_in may be NULL (zeros) and may
 * equal state_out (updated in place).
 */

/* Token-by-token recurrence. Replaces recurrent_gated_delta_rule,
 * motif/ops/gated_deltanet.py:26-59 (Dk <= 128, Dv <= 256). */
MB_API int motif_b200_gdn_recurrent(const void* q, const void* k, const void* v, const float* beta,
                             const float* g, const float* state_in, float* state_out, void* o,
                             int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                             const int64_t* strides, int dtype, void* stream);

/* Chunked form (chunk 64) fused in one kernel per (batch, head): intra-chunk UT transform,
 * inter-chunk state scan and output combine.  Replaces chunk_gated_delta_rule /
 * chunk_gated_delta_rule_triton, motif/ops/gated_deltanet.py:287-321 and :796-834
 * (Dk in {16,32,64}, Dv in {32,64,128}, Dv >= Dk). */
MB_API int motif_b200_gdn_chunk(const void* q, const void* k, const void* v, const float* beta,
                         const float* g, const float* state_in, float* state_out, void* o,
                         int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                         const int64_t* strides, int dtype, void* stream);

/* motif_b200_gdn_chunk with GatedRMSNorm fused into the output: each output row (token l
 * of head h) becomes rmsnorm(o) * onorm_w * silu(gate) with gate row
 * gate + (b*L + l)*gate_row_stride + h*gate_head_stride (token-major, Dv contiguous).
 * Replaces gdn_attn.py:197-209 (delta rule, o.to(dtype), o_norm(cat[o, gate])). */
MB_API int motif_b200_gdn_chunk_gated(const void* q, const void* k, const void* v, const float* beta,
                               const float* g, const float* state_in, float* state_out, void* o,
                               int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                               const int64_t* strides, const void* gate, int64_t gate_row_stride,
                               int64_t gate_head_stride, const void* onorm_w, float eps, int dtype,
                               void* stream);

/* Workspace bytes motif_b200_gdn_chunk_gated_ws needs for its two-kernel path (16-bit dtypes,
 * (Dk, Dv) in {(32,64), (64,64), (64,128)}); 0 when that path does not exist for the shape
 * (the call then runs the single fused kernel and needs no workspace). */
MB_API int64_t motif_b200_gdn_chunk_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                                             int dtype);

/* motif_b200_gdn_chunk_gated (gate may be NULL: plain motif_b200_gdn_chunk) with a
 * caller-provided device workspace of at least motif_b200_gdn_chunk_workspace_bytes bytes
 * (16-byte aligned).  With it the state-independent part of every chunk (gamma, the UT
 * transform W, U and the intra-chunk attention Aq) runs as one fully parallel kernel that
 * writes to the workspace, and only X = U - W S, the output and the state update walk the
 * chunks in order (motif/ops/gated_deltanet.py:137-177 + :287-321 split the same way).
 * workspace == NULL runs the fused kernel.  Same results contract as motif_b200_gdn_chunk_gated. */
MB_API int motif_b200_gdn_chunk_gated_ws(const void* q, const void* k, const void* v, const float* beta,
                                  const float* g, const float* state_in, float* state_out, void* o,
                                  int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                                  const int64_t* strides, const void* gate, int64_t gate_row_stride,
                                  int64_t gate_head_stride, const void* onorm_w, float eps, int dtype,
                                  void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ chord attention
 * Causal softmax attention with the gated geometric-decay bias
 *   logit(i,j) = (q_i.k_j * scale - alpha_h (|j - (q_start+i) - mu_h| + eps)^beta_h)
 *                * ssmax_h * log_n[b,i],   j <= q_start + i.
 * q,out: [B,H,L,D] dtype; k,v: [B,Hkv,S,D] dtype (H % Hkv == 0, head h reads kv head
 * h / (H/Hkv)); alpha,beta,mu,ssmax: [H] fp32; log_n: [B,L] fp32.
 * `strides` (elements), [14]: q(b,h,l) k(b,h,s) v(b,h,s) out(b,h,l) log_n(b,l).
 * `workspace` must hold motif_b200_chord_workspace_bytes(...) bytes (may be 0).
 * Replaces apply_chord_attention, motif/ops/chord_attention.py:1557-1625 (forward,
 * no autograd; D <= 128: tensor-core kernel for 16-bit dtypes and D in {16,32,64}, a
 * CUDA-core kernel otherwise). */
MB_API int64_t motif_b200_chord_workspace_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t L, int64_t S,
                                         int64_t D, int dtype);
MB_API int motif_b200_chord_attention(const void* q, const void* k, const void* v, const float* alpha,
                               const float* beta, const float* mu, const float* ssmax,
                               const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv,
                               int64_t L, int64_t S, int64_t D, int64_t q_start,
                               float softmax_scale, float eps, const int64_t* strides, int dtype,
                               void* workspace, int64_t workspace_bytes, void* stream);

/* motif_b200_chord_attention with an additive key bias: key_bias[b * key_bias_stride + s]
 * (fp32, natural-log units, -inf drops key s of sequence b) is added to every logit after the
 * ssmax * log n scaling, as ChordAttention applies `attention_mask` (a bool keep-mask as
 * 0 / -inf, or a float mask as is; motif/block/attention/chord_attn.py:347-356).  A row whose
 * keys are all dropped yields zeros (the reference's softmax yields NaN there). */
MB_API int motif_b200_chord_attention_masked(const void* q, const void* k, const void* v, const float* alpha,
                                      const float* beta, const float* mu, const float* ssmax,
                                      const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv,
                                      int64_t L, int64_t S, int64_t D, int64_t q_start, float scale,
                                      float eps, const int64_t* strides, const float* key_bias,
                                      int64_t key_bias_stride, int dtype, void* stream);

/* ------------------------------------------------------------------ attn-res / norms
 * Depth softmax over n_src (1..8) aligned [B,T,D] sources: logit_s = query . (weight *
 * rmsnorm(x_s)), h = sum_s softmax_s * x_s.  `src_strides` holds (batch, time) element
 * strides per source, [2*n_src]; weight, query: [D] dtype.
 * Replaces attn_res_block / _read_sources, motif/ops/attn_res.py:518-593. */
MB_API int motif_b200_attn_res(const void* const* sources, int n_src, const int64_t* src_strides,
                        const void* weight, const void* query, void* out, int64_t out_sb,
                        int64_t out_st, int64_t B, int64_t T, int64_t D, float eps, int dtype,
                        void* stream);

/* y = x * rsqrt(mean(x^2) + eps) * w over rows of N.  w may be NULL.
 * Replaces RMSNorm.forward, motif/ops/rms_norm.py:461-486. */
MB_API int motif_b200_rms_norm(const void* x, const void* w, void* y, int64_t M, int64_t N,
                        int64_t x_stride, int64_t y_stride, float eps, int dtype, void* stream);

/* y = rmsnorm(x[:, :N]) * w * silu(x[:, N:2N]) over rows of 2N.  w may be NULL.
 * Replaces GatedRMSNorm.forward, motif/ops/rms_norm.py:530-553. */
MB_API int motif_b200_gated_rms_norm(const void* x, const void* w, void* y, int64_t M, int64_t N,
                              int64_t x_stride, int64_t y_stride, float eps, int dtype,
                              void* stream);

/* y = x[:, :N] * silu(x[:, N:2N]).  Replaces SwiGLU.forward, motif/ops/swiglu.py:239-253. */
MB_API int motif_b200_swiglu(const void* x, void* y, int64_t M, int64_t N, int64_t x_stride,
                      int64_t y_stride, int dtype, void* stream);

/* ------------------------------------------------------------------ fused model kernels
 * These replace sequences of reference statements inside one layer; each cites them.
 * Token-major activations: row r = b*T + t, element stride 1 within a row.
 */

/* Attn-res read fused with the next RMSNorm: from n_src (1..8) aligned sources compute
 * h (softmax-weighted as motif_b200_attn_res when `query` != NULL, else the plain sum of
 * the sources), optionally store h to `h_out` (NULL = skip), and store
 * hn = h * rsqrt(mean(h^2) + eps) (no weight; norm weights are folded into the
 * following projection) to `hn_out`.  weight/query dtype.
 * Replaces decoder.py:189-207 (apply_block_attn_res + attn_norm / mlp_norm inputs) and
 * decoder.py:215 + motif.py:613 (block sum + final norm). */
MB_API int motif_b200_attn_res_norm(const void* const* sources, int n_src, int64_t src_row_stride,
                             const void* weight, const void* query, void* h_out,
                             void* hn_out, int64_t out_row_stride, int64_t rows, int64_t D,
                             float eps_src, float eps_out, int dtype, void* stream);

/* GDN input preparation over a [B,T] token block.  `proj` rows hold the concatenated
 * projections [q (H*Dk) | k (H*Dk) | v (H*Dv) | a (H) | b (H) | ...] (row stride
 * proj_stride).  Computes the causal depthwise conv (taps 4, weights [C][4] for the
 * C = H*(2Dk+Dv) q|k|v channels) over time with `conv_in` ([B,3,C] previous raw inputs,
 * NULL = zeros), SiLU, L2-normalised q*Dk^-0.5 and k, beta = sigmoid(b),
 * g = -exp(A_log) * softplus(a + dt_bias); writes q,k,v token-major ([B*T, H*D]),
 * beta/g as [B,T,H] fp32, and the last 3 raw inputs to `conv_out` ([B,3,C]; may alias
 * conv_in).  Replaces gdn_attn.py:116-136 and :183-197. */
MB_API int motif_b200_gdn_prep(const void* proj, int64_t proj_stride, const void* conv_w,
                        const void* A_log, const void* dt_bias, const void* conv_in,
                        void* conv_out, void* q, void* k, void* v, float* beta, float* g,
                        int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int dtype,
                        void* stream);

/* GDN prefill of a whole layer in ONE kernel (16-bit dtypes): motif_b200_gdn_prep's conv +
 * SiLU + L2 norms + beta/g computed on each chunk as it is staged, then the chunked delta
 * rule and the GatedRMSNorm epilogue of motif_b200_gdn_chunk_gated.  `proj` rows hold
 * [q | k | v | a | b | g | ...] (gate = g columns), row stride proj_stride (multiple of 8);
 * writes out[(b*T + t)*out_stride + h*Dv + j].  conv_in / conv_out: [B,3,C] (conv_out must
 * not alias conv_in); state_in may be NULL.  (Dk, Dv) in {(32,64), (64,64), (64,128)};
 * other shapes return MB_ERR_UNSUPPORTED (use gdn_prep + gdn_chunk_gated).
 * Replaces gdn_attn.py:183-209 for L > 1. */
MB_API int motif_b200_gdn_prefill(const void* proj, int64_t proj_stride, const void* conv_w,
                           const void* A_log, const void* dt_bias, const void* conv_in,
                           void* conv_out, const float* state_in, float* state_out,
                           const void* onorm_w, float eps, void* out, int64_t out_stride,
                           int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int dtype,
                           void* stream);

/* motif_b200_gdn_prefill with a caller-provided device workspace of at least
 * motif_b200_gdn_chunk_workspace_bytes(B, H, T, Dk, Dv, dtype) bytes (16-byte aligned).  With
 * it, (Dk, Dv) = (64, 128) runs as three kernels: the preparation (conv, SiLU, norms, beta, g)
 * fused into the fully parallel per-chunk UT transform, the state scan, and the gated norm;
 * other shapes (or workspace == NULL) run motif_b200_gdn_prefill.  Same results contract. */
MB_API int motif_b200_gdn_prefill_ws(const void* proj, int64_t proj_stride, const void* conv_w,
                              const void* A_log, const void* dt_bias, const void* conv_in,
                              void* conv_out, const float* state_in, float* state_out,
                              const void* onorm_w, float eps, void* out, int64_t out_stride,
                              int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int dtype,
                              void* workspace, int64_t workspace_bytes, void* stream);

/* One GDN decode step (T == 1) for a whole layer, fused: conv with the carried state,
 * SiLU, L2 norms, beta/g, the recurrent update of `state` ([B,H,Dk,Dv] fp32, in place)
 * and the gated RMSNorm of the output with gate columns `gate` (row stride proj_stride),
 * weight `onorm_w` [Dv]: writes out[B, H*Dv] (row stride out_stride).
 * Replaces gdn_attn.py:176-209 on the L == 1 path (recurrent_gated_delta_rule). */
MB_API int motif_b200_gdn_decode(const void* proj, int64_t proj_stride, const void* conv_w,
                          const void* A_log, const void* dt_bias, void* conv_state,
                          float* state, const void* gate, const void* onorm_w, void* out,
                          int64_t out_stride, int64_t B, int64_t H, int64_t Dk, int64_t Dv,
                          float eps, int dtype, void* stream);
/* motif_b200_gdn_decode plus the decoder's SwiGLU MLP activation in the same launch:
 * act[b, :hid] = gu[b, :hid] * silu(gu[b, hid:2 hid]) (motif/ops/swiglu.py:252-253), rows of
 * gu / act strided by gu_stride / act_stride elements.  The two are independent (both read
 * the packed projection row), so extra CTAs of the GDN launch compute the activation; when
 * that is not possible (fp32, unaligned rows, a shape without the split kernel) a separate
 * SwiGLU launch follows, with the same results.  Replaces decoder.py:203-207's GDN step and
 * mlp.py's activation. */
MB_API int motif_b200_gdn_decode_swiglu(const void* proj, int64_t ps, const void* conv_w, const void* A_log,
                                 const void* dt_bias, void* conv_state, float* state, const void* gate,
                                 const void* onorm_w, void* out, int64_t os, int64_t B, int64_t H,
                                 int64_t Dk, int64_t Dv, float eps, const void* gu, int64_t gu_stride,
                                 void* act, int64_t act_stride, int64_t hid, int dtype, void* stream);

/* Chord input preparation: per token, RMSNorm each q head (weight qn_w [D]) and each k
 * head (kn_w [D]) of `proj` rows [q (H*D) | k (Hkv*D) | v (Hkv*D) | ...]; writes q
 * token-major [B*T, H*D] and appends k, v into the cache buffers k_cache/v_cache
 * ([B,Hkv,cap,D]) at positions pos .. pos+T-1, where pos = *pos_dev if pos_dev != NULL
 * else pos_host.  Replaces chord_attn.py:256-270 (projections' norms + KVLayerCache.update). */
MB_API int motif_b200_chord_prep(const void* proj, int64_t proj_stride, const void* qn_w,
                          const void* kn_w, void* q, void* k_cache, void* v_cache, int64_t cap,
                          const int32_t* pos_dev, int64_t pos_host, int64_t B, int64_t T,
                          int64_t H, int64_t Hkv, int64_t D, float eps, int dtype, void* stream);
/* motif_b200_chord_prep plus the decoder's SwiGLU MLP activation over the B*T rows in the
 * same launch (as motif_b200_gdn_decode_swiglu; a separate SwiGLU launch follows when the
 * vector kernel cannot run). */
MB_API int motif_b200_chord_prep_swiglu(const void* proj, int64_t proj_stride, const void* qn_w,
                                 const void* kn_w, void* q, void* k_cache, void* v_cache, int64_t cap,
                                 const int32_t* pos_dev, int64_t pos_host, int64_t B, int64_t T, int64_t H,
                                 int64_t Hkv, int64_t D, float eps, const void* gu, int64_t gu_stride,
                                 void* act, int64_t act_stride, int64_t hid, int dtype, void* stream);

/* Chord decode/short-query attention over a cache whose length is read on the device:
 * S = *len_dev (+ T new tokens already appended), q_start = S - T.  Same math as
 * motif_b200_chord_attention; q token-major [B*T, H*D], out token-major (out_stride).
 * `workspace` >= motif_b200_chord_decode_workspace_bytes(B,H,T,D,max_splits).
 * Replaces the L <= 8 use of apply_chord_attention from chord_attn.py:295-313. */
MB_API int64_t motif_b200_chord_decode_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t D,
                                                int max_splits);
MB_API int motif_b200_chord_decode(const void* q, const void* k_cache, const void* v_cache, int64_t cap,
                            const int32_t* len_dev, int64_t len_host, const float* alpha,
                            const float* beta, const float* mu, const float* ssmax,
                            void* out, int64_t out_stride, int64_t B, int64_t H, int64_t Hkv,
                            int64_t T, int64_t D, float softmax_scale, float eps,
                            int max_splits, void* workspace, int64_t workspace_bytes, int dtype,
                            void* stream);

/* motif_b200_chord_decode with the additive key bias of motif_b200_chord_attention_masked
 * (row stride key_bias_stride >= the attended length). */
MB_API int motif_b200_chord_decode_masked(const void* q, const void* k_cache, const void* v_cache, int64_t cap,
                                   const int32_t* len_dev, int64_t len_host, const float* alpha,
                                   const float* beta, const float* mu, const float* ssmax, void* out,
                                   int64_t out_stride, int64_t B, int64_t H, int64_t Hkv, int64_t T, int64_t D,
                                   float scale, float eps, int max_splits, const float* key_bias,
                                   int64_t key_bias_stride, void* workspace, int64_t workspace_bytes,
                                   int dtype, void* stream);

/* motif_b200_chord_decode without a caller-provided workspace: for callers that cannot
 * allocate device memory (a runtime bound through a plain C FFI with no CUDA allocator of
 * its own, or a serving loop that must not call cudaMalloc between steps).  The split
 * partials go to one fixed 8 MiB device array inside the library instead; requests whose
 * motif_b200_chord_decode_workspace_bytes(B, H, T, D, max_splits) exceeds 8 MiB fail with
 * MB_ERR_SHAPE.  The array is shared by every call on a device: calls that overlap on the
 * GPU (e.g. on two streams at once) race and must be serialised by the caller.  The first
 * call on each device looks up the array's device address (with that device current); make
 * that first call before any stream capture.  Allocates nothing.
 * No counterpart in the reference: an addition of this library. */
MB_API int motif_b200_chord_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                    int64_t cap, const int32_t* len_dev, int64_t len_host,
                                    const float* alpha, const float* beta, const float* mu,
                                    const float* ssmax, void* out, int64_t out_stride, int64_t B,
                                    int64_t H, int64_t Hkv, int64_t T, int64_t D,
                                    float softmax_scale, float eps, int max_splits, int dtype,
                                    void* stream);

/* Number of CTAs whose bounded wait for a tensor / bulk copy or an MMA ran out since the last
 * call (Chord decode: motif_b200_chord_decode / _noalloc; tensor-core Chord prefill:
 * motif_b200_chord_attention; the GDN state scan of motif_b200_gdn_chunk_gated_ws); such a
 * CTA abandons its work (a decode split contributes nothing, a prefill tile's rows or a
 * scan's outputs are left unwritten) instead of hanging.  The counter is cleared.
 * Synchronous (copies from device memory).  Expected to stay 0.  No counterpart in the
 * reference. */
MB_API int motif_b200_wait_timeouts(uint32_t* count);

/* Decode-sized products Y[M, N] = X[M, K] . W[N, K]^T, 1 <= M <= 64, 16-bit operands, fp32
 * accumulation, on a weight packed once in tensor-core fragment order.
 *
 * motif_b200_skinny_packed_bytes(N, K): size of the packed copy of W (N rounded up to 32
 *   features; -1 if K is not a positive multiple of 16).
 * motif_b200_skinny_pack: W [N, K] (row stride ldw elements, even, W 4-byte aligned) into
 *   `packed` (16-byte aligned, motif_b200_skinny_packed_bytes(N, K) bytes).  Asynchronous on
 *   `stream`.  Pack again after changing W.
 * motif_b200_skinny_gemm: Y (row stride ldy; N and ldy multiples of 4, Y 8-byte aligned) from
 *   X (row stride ldx, a multiple of 8, 16-byte aligned) and the packed W; K a multiple of 16.
 *   Each warp loads its weight blocks straight from HBM into the registers the MMA reads
 *   before waiting on the previous kernel (programmatic dependent launch); K is split across
 *   the warps of a CTA and across the CTAs of a cluster (at most 8), with the partial tiles
 *   summed in a fixed order, so results are deterministic.  k_warps (1, 2 or 4) and split_k
 *   (1 .. 8) force the split; 0 lets the library choose.  Other shapes: MB_ERR_UNSUPPORTED.
 * Replaces the decode-time nn.Linear products (gdn_attn.py:88-94, chord_attn.py:88-96,
 * mlp.py:52-53, the decoders' o_proj / down_proj, motif.py lm_head) that cuBLAS runs as
 * weight-bandwidth-bound small-M GEMMs. */
MB_API int64_t motif_b200_skinny_packed_bytes(int64_t N, int64_t K);
MB_API int motif_b200_skinny_pack(const void* w, int64_t ldw, int64_t N, int64_t K, void* packed, int dtype,
                                  void* stream);
MB_API int motif_b200_skinny_gemm(const void* x, int64_t ldx, const void* packed, void* y, int64_t ldy, int64_t M,
                                  int64_t N, int64_t K, int k_warps, int split_k, int dtype, void* stream);

/* Decode-sized products on the tensor cores: Y[M, N] = X[M, K] . W[N, K]^T for 1 <= M <= 64
 * (the one-GPU decode batch), 16-bit operands, fp32 accumulation, on the weight itself (no
 * packing).  X and W rows 16-byte aligned (ldx, ldw multiples of 8), K a multiple of 64; Y row
 * stride ldy, N and ldy multiples of 4, Y 8-byte aligned.  Each CTA streams one 128-feature
 * tile of W over a run of K by tiled TMA, requested before the kernel waits on the previous
 * kernel (programmatic dependent launch), into tcgen05.mma with a TMEM accumulator; K is split
 * across the CTAs of a cluster (at most 8) whose fp32 partial tiles are exchanged by bulk
 * copies between their shared memories and summed in a fixed order (deterministic).  split_k
 * (1 .. 8) forces the split; 0 lets the library choose.  Asynchronous on `stream`.
 * Replaces the same decode-time nn.Linear products as motif_b200_skinny_gemm
 * (gdn_attn.py:88-94, chord_attn.py:88-96, mlp.py:52-53, the decoders' o_proj / down_proj). */
MB_API int motif_b200_skinny_gemm_tc(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                                     int64_t M, int64_t N, int64_t K, int split_k, int dtype, void* stream);
/* motif_b200_skinny_gemm_tc with the Chord decoder's parallel residual in the epilogue:
 *   y = round(round(a * round(sigmoid(g))) + round(x . w^T))
 * (the MLP's down projection plus the gated attention output; a [M, N] is the o_proj output,
 * g [M, N] the gate projection, both 16-bit with rows 8-byte aligned and strides multiples of
 * 4; y must not overlap them).  Bit-identical to motif_b200_skinny_gemm_tc followed by
 * motif_b200_gate_residual.  Replaces chord_attn.py:254,313 (o_proj(out) * G) and the parallel
 * residual of decoder.py:208 for decode-sized batches. */
MB_API int motif_b200_skinny_gemm_tc_add_gated(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                               const void* a, int64_t lda, const void* g, int64_t ldg, void* y,
                                               int64_t ldy, int64_t M, int64_t N, int64_t K, int split_k,
                                               int dtype, void* stream);
/* The Chord decoder's whole tail in one launch on the tensor-core decode GEMM:
 *   y = round(round(round(x1 . w1^T) * round(sigmoid(g))) + round(x2 . w2^T))
 * with x1 [M, K1] the attention output and w1 [N, K1] o_proj, x2 [M, K2] the MLP activation
 * and w2 [N, K2] down_proj, g [M, N] the gate (rows 8-byte aligned, stride a multiple of 4).
 * The cluster's ranks split the K of both products; each product's partials are summed apart
 * in rank order (deterministic).  Same operand rules as motif_b200_skinny_gemm_tc; y must not
 * overlap the inputs.  Replaces chord_attn.py:254,313 (o_proj(out) * G) with the MLP's down
 * projection (mlp.py:63) and the parallel residual (decoder.py:208) for decode-sized batches. */
MB_API int motif_b200_skinny_gemm_tc_chord_tail(const void* x1, int64_t ldx1, const void* w1, int64_t ldw1,
                                                int64_t K1, const void* x2, int64_t ldx2, const void* w2,
                                                int64_t ldw2, int64_t K2, const void* g, int64_t ldg, void* y,
                                                int64_t ldy, int64_t M, int64_t N, int dtype, void* stream);

/* ------------------------------------------------------------------ backward (training)
 * Gradients of the three hot-path ops, fp32 arithmetic on CUDA cores (16-bit inputs widened on
 * load), asynchronous on `stream`.
 *
 * motif_b200_chord_backward: dq [B,H,L,D], dk / dv [B,Hkv,S,D] (summed over each kv head's
 *   query heads) from q, k, v, the forward output `out` and `dout`, with the forward's
 *   arguments; `strides` holds the (b, head, t) element strides of q, k, v, out, dout, dq, dk,
 *   dv and the (b, t) strides of log_n (26 values; unit inner strides).  Each row's
 *   log-sum-exp is recomputed.  `param_partials` [B][H][ceil(L/32)][4] fp64 receives per-tile
 *   partial gradients of alpha, beta, mu, ssmax (the caller sums over batch and tiles).
 *   `workspace`: motif_b200_chord_backward_workspace_bytes(B, H, L), 16-byte aligned.
 *   D in {16, 32, 64, 128}.  Replaces `_chord_backward_impl` / `_chord_bwd_dq_kernel` /
 *   `_chord_bwd_dkdv_kernel` (motif/ops/chord_attention.py:518-958, 1348-1445).
 * motif_b200_attn_res_backward: the gradient of every source (d_sources, same layout: rows of
 *   D elements, row stride `row_stride`) and, in z_partials [partial_rows][D] fp32, partial
 *   sums Z of which dquery = weight * sum(Z) and dweight = query * sum(Z); one launch of
 *   `partial_rows` CTAs.  Replaces `_AttnResFunction.backward` (motif/ops/attn_res.py:188-364,
 *   425-463).
 * motif_b200_gdn_backward: dq, dk [B,H,L,Dk], dv [B,H,L,Dv], dbeta, dg [B,H,L] and (when
 *   d_state_in is not null) the initial state's gradient, from grad_out [B,H,L,Dv] and
 *   grad_state (the final state's gradient, or null); all fp32 and contiguous.  The states are
 *   rebuilt from checkpoints every 64 steps in `workspace`
 *   (motif_b200_gdn_backward_workspace_bytes).  (Dk, Dv) in {(16,32), (32,32), (32,64),
 *   (64,64), (64,128), (128,128)}.  Replaces the backward of `_PrepareChunksFunction` and
 *   `_FusedScanFunction` (motif/ops/gated_deltanet.py:180-284, 427-611, 726-765). */
MB_API int64_t motif_b200_chord_backward_workspace_bytes(int64_t B, int64_t H, int64_t L);
MB_API int motif_b200_chord_backward(const void* q, const void* k, const void* v, const void* out, const void* dout,
                                     const float* alpha, const float* beta, const float* mu, const float* ssmax,
                                     const float* log_n, void* dq, void* dk, void* dv, int64_t B, int64_t H,
                                     int64_t Hkv, int64_t L, int64_t S, int64_t D, int64_t q_start, float scale,
                                     float eps, const int64_t* strides, void* workspace, int64_t workspace_bytes,
                                     double* param_partials, int dtype, void* stream);
MB_API int motif_b200_attn_res_backward(const void* const* sources, void* const* d_sources, int n_src, int64_t rows,
                                        int64_t row_stride, int64_t D, const void* weight, const void* query,
                                        float eps, const void* grad_out, int64_t grad_stride, float* z_partials,
                                        int64_t partial_rows, int dtype, void* stream);
MB_API int64_t motif_b200_gdn_backward_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv);
MB_API int motif_b200_gdn_backward(const float* q, const float* k, const float* v, const float* beta, const float* g,
                                   const float* state_in, const float* grad_out, const float* grad_state, float* dq,
                                   float* dk, float* dv, float* dbeta, float* dg, float* d_state_in, int64_t B,
                                   int64_t H, int64_t L, int64_t Dk, int64_t Dv, void* workspace,
                                   int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ dense projections
 * Y = X . W^T for 16-bit X [M, K] and W [N, K] (row strides ldx / ldw in elements, multiples of
 * 8, 16-byte aligned; K a multiple of 64, else MB_ERR_UNSUPPORTED), fp32 accumulation on the
 * tensor cores (tcgen05, one persistent CTA per SM), output in the input dtype.  fp32 models
 * keep the library GEMM (these kernels are 16-bit only: MB_ERR_UNSUPPORTED).
 * Replaces the prefill-time nn.Linear products of the reference's layers
 * (block/attention/gdn_attn.py:88-94, chord_attn.py:88-96, block/mlp.py:52-53,
 * model/motif.py:184 lm_head), each with the elementwise step that follows it fused in. */
MB_API int motif_b200_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                           int64_t M, int64_t N, int64_t K, int dtype, void* stream);
/* The packed input projection of a decoder with its MLP activation fused: W holds n_plain
 * projection rows, then the MLP's gate_up rows regrouped in blocks of 256 (128 value rows, then
 * the 128 gate rows of the same hidden units; hid a multiple of 128).  y[:, :n_plain] = X . W[:
 * n_plain]^T, and act[:, :hid] = SwiGLU of the gate_up product with the reference's rounding
 * points: round(round(v) * round(silu(round(g)))) (block/mlp.py:52-53 + ops/swiglu.py:252-253).
 * n_plain or hid may be 0. */
MB_API int motif_b200_gemm_proj_swiglu(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M,
                                       int64_t K, int64_t n_plain, void* y, int64_t ldy, int64_t hid, void* act,
                                       int64_t ld_act, int dtype, void* stream);
/* The gated delta-net layer's packed input projection with the layer's preparation and the MLP
 * activation in its epilogue.  W rows: q (H*dk) | k (H*dk) | v (H*dv) | a (H) | b (H) |
 * g (H*dv) | gate_up (2*hid, regrouped as for motif_b200_gemm_proj_swiglu).  X is [B*T, K], the
 * rows of B sequences of T tokens.  Outputs (token-major, contiguous): q, k [B*T, H*dk] after the
 * causal depthwise conv (kernel 4, carried state conv_in [B, 3, C] or zeros; C = H*(2dk+dv)),
 * SiLU and the per-head L2 norm (q also times dk^-1/2); v [B*T, H*dv] after conv + SiLU;
 * beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) as fp32 [B*T, H]; gate [B*T, H*dv]
 * (the g projection, for the gated norm); act (row stride ld_act) the SwiGLU; conv_out
 * [B, 3, C] (optional) the raw inputs of each sequence's last three tokens.  Rounding points as
 * the reference's bf16 layer.  dk = 64, dv a multiple of 32, H <= 16, T >= 3, hid a multiple
 * of 128.  Replaces gdn_attn.py:88-94 (projections), :116-136 (_conv), :183-197 (normalise,
 * beta, g) and block/mlp.py:52-53. */
MB_API int motif_b200_gemm_gdn_prep(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t B, int64_t T,
                                    int64_t K, int64_t H, int64_t dk, int64_t dv, int64_t hid, const void* conv_w,
                                    const void* A_log, const void* dt_bias, const void* conv_in, void* conv_out,
                                    void* q, void* k, void* v, float* beta, float* g, void* gate, void* act,
                                    int64_t ld_act, int dtype, void* stream);
/* The Chord output projection with the gate and the parallel residual fused:
 * out = round(round(round(X . W^T) * round(sigmoid(gate))) + res) over [M, N]; out may alias res.
 * Replaces chord_attn.py:254,313 (o_proj(out) * G) and decoder.py:208 (attn + mlp). */
MB_API int motif_b200_gemm_gate_residual(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                         const void* gate, int64_t ldg, const void* res, int64_t ldr, void* out,
                                         int64_t ldo, int64_t M, int64_t N, int64_t K, int dtype, void* stream);

/* out = a * sigmoid(gate) + m over [rows, N] (row strides given).
 * Replaces chord_attn.py:254,313 (o_proj(out) * G) + decoder.py:208 (attn + mlp). */
MB_API int motif_b200_gate_residual(const void* a, int64_t a_stride, const void* gate,
                             int64_t gate_stride, const void* m, int64_t m_stride, void* out,
                             int64_t out_stride, int64_t rows, int64_t N, int dtype, void* stream);

/* Greedy next token: ids[r] = argmax over V of logits row r (first maximum), int64.
 * Replaces ModelOutput.next_token's argmax, motif/model/motif.py:92-98. */
MB_API int motif_b200_argmax(const void* logits, int64_t rows, int64_t V, int64_t row_stride,
                      int64_t* ids, int dtype, void* stream);

/* End of a CUDA-graph decode step in one launch: tokens[*step_idx, :B] = ids[:B] (a
 * [max_steps, B] int64 log; skipped when *step_idx is outside [0, max_steps)), then
 * *step_idx += 1 and lens[0 .. nlens) += 1 (int32 cache lengths, nlens <= 64).  Replaces
 * the token append and position advance of the reference's generation loop
 * (motif/model/generate.py:138-171) inside the captured step. */
MB_API int motif_b200_decode_advance(const int64_t* ids, int64_t B, int64_t* tokens, int64_t max_steps,
                              int64_t* step_idx, int32_t* lens, int64_t nlens, void* stream);

/* One sampled token per row (Sampler.__call__, motif/model/sampler.py:151-219, without the
 * grammar constraint, whose mask the caller applies to the logits first): repetition penalty
 * over the distinct ids of history[r, :hist_len] (negative ids ignored) -> temperature
 * (x / max(T, 1e-5) when T != 1) -> top-k (top_k <= 0: off) -> top-p (p outside (0, 1):
 * off) -> softmax -> draw.  The draw takes uniforms[r] in [0, 1) when `uniforms` is given,
 * else Philox4x32-10 with key `seed` and counter (r, 0, offset + *offset_dev) (offset_dev may
 * be NULL); the token is the first index whose inclusive cumulative probability exceeds
 * u * total.  out: B int64 (-1 for a row with no finite logit); probs_out (optional, fp32
 * [B, probs_ld]) receives the final distribution.  V <= 53248 (MB_ERR_UNSUPPORTED above).
 * `logits` has row stride ld (elements) and dtype `dtype`. */
MB_API int motif_b200_sample(const void* logits, int64_t ld, int64_t B, int64_t V, const int64_t* history,
                      int64_t hist_ld, int64_t hist_len, float repetition_penalty, float temperature,
                      int64_t top_k, float top_p, const float* uniforms, uint64_t seed, uint64_t offset,
                      const int64_t* offset_dev, int64_t* out, float* probs_out, int64_t probs_ld,
                      int dtype, void* stream);

/* Testing hook, no counterpart in the reference: forces one of the kernels that a shape or
 * dtype also selects onto calls the default routing sends elsewhere, so tests can compare
 * two kernels on the same inputs.  Every knob is off at load; the setting is process-wide
 * and read at each launch.  Not for production use.
 *   MB_FORCE_CHORD_MMA_SYNC  16-bit D = 64 Chord prefill on the mma.sync kernel (D = 16 / 32's)
 *   MB_FORCE_DECODE_SCALAR   16-bit D = 64 Chord decode on the CUDA-core kernel (fp32's)
 *   MB_FORCE_GDN_PRECISE     16-bit chunked delta rule on the 3xTF32 kernel (fp32's)
 *   MB_FORCE_GDN_FUSED       16-bit chunked delta rule with a workspace on the single fused
 *                            kernel (the no-workspace path)
 *   MB_FORCE_GDN_WIDE        the split path's state scan on 64-column value slices even for small
 *                            batches (which take 32-column slices; the results are identical) */
enum {
  MB_FORCE_CHORD_MMA_SYNC = 0,
  MB_FORCE_DECODE_SCALAR = 1,
  MB_FORCE_GDN_PRECISE = 2,
  MB_FORCE_GDN_FUSED = 3,
  MB_FORCE_GDN_WIDE = 4,
  MB_FORCE_COUNT = 5
};
MB_API int motif_b200_testing_force(int knob, int value);

/* Token embedding gather: out[r] = table[ids[r]] ([V, D] rows), motif/model/motif.py:604. */
MB_API int motif_b200_embed(const int64_t* ids, const void* table, void* out, int64_t rows, int64_t D,
                     int64_t V, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOTIF_B200_H */
