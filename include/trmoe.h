/* trmoe.h: the C ABI of libtrmoe.so, Trochilus's OLMoE Mixture-of-Experts layer on an NVIDIA B200.
 *
 * Two levels, both plain C (pointers and sizes; no CUDA or torch types in the signatures):
 *
 *  1. The layer hook, modelled on Trochilus's GPU attention backend (src/backend/gpu_attn.h:32-74): a
 *     tr_gpu_moe holds every layer's router and experts resident in HBM, uploaded once from the host
 *     GGUF bytes, and runs one MoE layer per call from the normed FFN input to the residual add. It
 *     replaces forward_layer's block from the router matmul to the mix (src/models/olmoe.c:1845-1933).
 *
 *  2. The kernel level, the same names and arguments as Trochilus's quantized-matmul API
 *     (src/kernels/kernels.h:239-300, 342-350): tr_matmul, tr_matmul_grouped(_s), tr_softmax,
 *     tr_swiglu. Pointers are the caller's host memory as in the reference; a weight is uploaded the
 *     first time its data pointer is seen and then read from HBM (the pointer must stay valid and its
 *     bytes unchanged, as the reference's expert store slots are). The pool argument is ignored.
 *
 * Numerics: every result is bit for bit Trochilus's scalar definition (the 16-lane contract for F32,
 * BF16, Q8_0 and Q6_K rows; Q4_K's exact-integer definition; the correctly rounded exp; the id-ordered
 * combine), for every token count.
 *
 * Conventions kept from gpu_attn.h: int results are 0 on success and -1 on failure; creation returns
 * NULL with a message in (err, err_len); one context, one thread at a time. There is no CPU fallback:
 * a failure is an error. The void kernel-level calls have no return code in the reference; on a
 * failure they print the reason to stderr, record the message that trmoe_last_error() returns and set
 * every output float the call owns to a quiet NaN, so that nothing computed from it passes for a result.
 * With TRMOE_ABORT_ON_ERROR=1 in the environment they abort() the process instead. */
#ifndef TRMOE_H
#define TRMOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TRMOE_API __attribute__((visibility("default")))
#else
#define TRMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ggml tensor type numbers (Trochilus src/format/gguf.h:16-27); the supported subset */
enum { TRMOE_F32 = 0, TRMOE_F16 = 1, TRMOE_Q8_0 = 8, TRMOE_Q4_K = 12, TRMOE_Q6_K = 14, TRMOE_BF16 = 30 };

/* ---------------------------------------------------------------------------------------------
 * 1. The layer hook */

typedef struct tr_gpu_moe tr_gpu_moe;

typedef struct {
    int64_t n_layers;   /* layers held */
    int64_t n_expert;   /* experts per layer (<= 64) */
    int64_t n_used;     /* experts per token (<= 32, <= n_expert) */
    int64_t n_embd;     /* hidden size H: a multiple of 256 (OLMoE: 2048) */
    int64_t n_ff;       /* expert intermediate size F: a multiple of 256 (OLMoE: 1024) */
    int32_t norm_topk;  /* 1: the k weights renormalised to sum 1 (OLMoE: 0) */
    int32_t router_type; /* F32 or BF16 */
    int32_t gate_type;   /* Q8_0 or Q4_K (gate and up share it) */
    int32_t down_type;   /* Q8_0, Q4_K or Q6_K */
    int64_t max_tokens;  /* the most tokens one call passes */
} tr_gpu_moe_config;

/* Replaces: tr_gpu_attn_create (src/backend/gpu_attn.h:46-47) as the model's GPU context for the MoE
 * layer. Device `device` (CUDA ordinal); the layers are set by tr_gpu_moe_set_layer. NULL with a
 * message when the shape or a type is not supported, or HBM is short. */
TRMOE_API tr_gpu_moe *tr_gpu_moe_create(const tr_gpu_moe_config *cfg, int device, char *err, size_t err_len);
/* Replaces: tr_gpu_attn_free (src/backend/gpu_attn.h:48). NULL: nothing. */
TRMOE_API void tr_gpu_moe_free(tr_gpu_moe *m);
/* Replaces: tr_gpu_attn_bytes (src/backend/gpu_attn.h:50): bytes of HBM a context of cfg holds. */
TRMOE_API uint64_t tr_gpu_moe_bytes(const tr_gpu_moe_config *cfg);

/* Uploads layer `layer`'s weights from host GGUF bytes, replacing the reference's expert-store slots
 * (src/models/olmoe.c:2146-2186; the tr_mat views of olmoe.c:466-472): router = n_expert rows of
 * n_embd (ffn_gate_inp); router_bias = NULL or n_expert floats added to every logit (a benchmark
 * extension, not in the reference); gate[e], up[e] = n_ff rows of n_embd; down[e] = n_embd rows of
 * n_ff. Returns when the bytes are in HBM. 0, or -1 with a message. */
TRMOE_API int tr_gpu_moe_set_layer(tr_gpu_moe *m, int64_t layer, const void *router, const float *router_bias,
                         const void *const *gate, const void *const *up, const void *const *down, char *err,
                         size_t err_len);

/* The model loader (the rank-4 next step beyond the MoE block): an OLMoE GGUF file (versions 2 and 3) straight into
 * the context's resident layout, in place of the reference's load (src/models/olmoe.c:541-641, 895-925) and its
 * expert store (src/memory/experts.h): every layer's experts live in HBM, none on the host.
 * tr_gpu_moe_config_from_gguf fills cfg's n_layers, n_expert, n_used, n_embd, n_ff, norm_topk and the three types
 * from the file's olmoe.* metadata and its ffn_gate_inp / ffn_*_exps tensors (max_tokens is left as the caller set
 * it), and *rms_eps (optional) from olmoe.attention.layer_norm_rms_epsilon. router_type is BF16 when every router is
 * BF16 or an F32 whose values are all bfloat16 (the reference keeps those as BF16, olmoe.c:391), else F32. A file
 * whose layers use different expert types is refused (a context takes one gate/up type and one down type). Every
 * count, length and offset is checked against the file's size. Host only. 0, or -1 with a message. */
TRMOE_API int tr_gpu_moe_config_from_gguf(const char *path, tr_gpu_moe_config *cfg, float *rms_eps, char *err,
                                          size_t err_len);
/* Sets every layer of m from the file: tr_gpu_moe_set_layer with the router (narrowed to BF16 or widened to F32 as
 * the context's type asks) and the 64 experts' slices of each stacked tensor, and tr_gpu_moe_set_ffn_norm with the
 * layer's ffn_norm and the file's epsilon. The file must give m's configuration (tr_gpu_moe_config_from_gguf's).
 * The file is mapped read-only while the call runs. 0, or -1 with a message. */
TRMOE_API int tr_gpu_moe_load_gguf(tr_gpu_moe *m, const char *path, char *err, size_t err_len);

/* Replaces: forward_layer's MoE block from the router to the mix (src/models/olmoe.c:1845-1933), the
 * hook sitting where tr_gpu_attn_decode sits for the attention (olmoe.c:1790-1797).
 * normed: n_tok rows of n_embd (the ffn_norm output); x_inout: the residual stream, n_tok rows of
 * n_embd, to which the layer's output is added. sel_id_out, sel_w_out (optional): the n_tok * n_used
 * experts (increasing id per token) and their weights. Host memory (pinned or not). Returns when x
 * holds the result. 0, or -1 on a CUDA error or a bad argument.
 * Pinned x (page-locked and mapped, as the reference's gpu_attn.h:11-14 in/out buffers) and calls of up to
 * 16 tokens without sel outputs: the GPU reads and writes x in place and posts its completion to pinned
 * memory the call polls (no copy of x, no stream synchronisation); otherwise x is copied in and out. */
TRMOE_API int tr_gpu_moe_layer(tr_gpu_moe *m, int64_t layer, const float *normed, int64_t n_tok, float *x_inout,
                     int64_t *sel_id_out, float *sel_w_out);

/* ffn_norm moved into the hook (the rank-1 next step beyond the MoE block): the FFN sub-block of forward_layer
 * from its ffn_norm to the mix (src/models/olmoe.c:1834-1933), so that the engine passes the residual stream and
 * no normed rows cross the host link.
 * tr_gpu_moe_set_ffn_norm replaces the layer's ffn_norm tensor view (olmoe.c:1836, layer->ffn_norm: n_embd floats)
 * and the model's epsilon (olmoe.c:556, olmoe.attention.layer_norm_rms_epsilon). 0, or -1 with a message. */
TRMOE_API int tr_gpu_moe_set_ffn_norm(tr_gpu_moe *m, int64_t layer, const float *weight, float eps, char *err,
                                      size_t err_len);

/* Replaces: olmoe.c:1834-1933 (norm_body's tr_rmsnorm per token, src/kernels/kernels.c:1351-1360, then the MoE
 * block as tr_gpu_moe_layer). x_inout: the residual stream, n_tok rows of n_embd, normalised into the layer's
 * input and then given the layer's output. normed_out (optional): the n_tok normalised rows. Host memory, as
 * tr_gpu_moe_layer (pinned x: the same in-place road). 0, or -1 with a message (also when the layer has no
 * ffn_norm weight). */
TRMOE_API int tr_gpu_moe_ffn(tr_gpu_moe *m, int64_t layer, int64_t n_tok, float *x_inout, float *normed_out,
                             int64_t *sel_id_out, float *sel_w_out);

/* Optional device outputs of tr_gpu_moe_layer_dev (any field NULL: not written) */
typedef struct {
    float *logits;      /* [n_tok][n_expert] router logits (after the bias) */
    int64_t *sel_id;    /* [n_tok * n_used] */
    float *sel_w;       /* [n_tok * n_used] */
    int64_t *offsets;   /* [n_expert + 1] segment starts of the grouped order */
    int64_t *place;     /* [n_tok * n_used] grouped position of each (token, slot) row */
    float *ffn_out;     /* [n_tok][n_embd] the layer's output before the residual add */
} tr_gpu_moe_outputs;

/* Expert parallelism (no counterpart in the reference, which runs on one host; the plan is its routing, counting
 * sort and mix, src/models/olmoe.c:1845-1933, split across GPUs that hold E / n_ranks experts each). A rank passes
 * NULL for the gate, up and down pointers of experts it does not hold to tr_gpu_moe_set_layer. Per layer call:
 *   1. tr_gpu_moe_layer_part(part 0) with sel_id / sel_w outputs routes the rank's own tokens;
 *   2. tr_gpu_moe_ep_pack groups the rank's R = n_tok * n_used (token, slot) rows by destination rank (expert / (E /
 *      n_ranks)), stably: d_send_rows (rows x n_embd f32), d_send_ids (int32 expert ids), d_send_counts[n_ranks],
 *      d_place[j] = row j's position in that order; d_scratch: 72 + R int32. cap = 0: the rows packed (R of them);
 *      cap >= R: destination d's rows at d cap .. (n_ranks x cap rows, unused ids -1), so that an all-to-all of equal
 *      splits needs no counts on the host;
 *   3. the caller exchanges counts, rows and ids (NCCL all-to-all);
 *   4. tr_gpu_moe_experts_dev computes the expert FFN (gate/up, SwiGLU, down; the exact definitions) of n_rows rows
 *      that arrived in any order with their expert ids, into d_out (n_rows x n_embd), in arrival order (a row whose id
 *      is out of range, the padding, gets no expert: its output row is left as it was or zeroed). Calls of up to 64
 *      rows and at most the context's max_tokens run as one fused kernel, so create a rank's context with
 *      max_tokens >= the most rows it receives (n_ranks x cap in the padded exchange);
 *   5. the caller sends the outputs back;
 *   6. tr_gpu_moe_ep_combine: x[t] += sum over slots in expert-id order of sel_w[t][slot] * d_back[place[t k + slot]]
 *      (and ffn_out, if not NULL).
 * The result is bit for bit the one-GPU layer's. Device pointers; `stream` NULL: the context's stream. 0 or -1. */
TRMOE_API int tr_gpu_moe_ep_pack(tr_gpu_moe *m, const int64_t *d_sel_id, int64_t n_tok, int32_t n_ranks, int64_t cap,
                                 const float *d_normed, float *d_send_rows, int32_t *d_send_ids, int32_t *d_send_counts,
                                 int32_t *d_place, int32_t *d_scratch, void *stream);
TRMOE_API int tr_gpu_moe_experts_dev(tr_gpu_moe *m, int64_t layer, const float *d_rows, const int32_t *d_ids,
                                     int64_t n_rows, float *d_out, void *stream);
TRMOE_API int tr_gpu_moe_ep_combine(tr_gpu_moe *m, const float *d_sel_w, const int32_t *d_place, const float *d_back,
                                    int64_t n_tok, float *d_x, float *d_ffn_out, void *stream);

/* Expert parallelism over peer memory (NVLink stores between the ranks' GPUs, no NCCL on the data path; a B200
 * replacement for the all-to-alls above, same plan and the same bit-for-bit result). Each rank's context owns an
 * exchange region for n_ranks sources of cap rows each (cap >= n_tok x n_used of every call). Set-up, once:
 * tr_gpu_moe_ep_peer_region makes the region and writes its CUDA IPC handle (TRMOE_IPC_HANDLE_BYTES) to
 * ipc_handle_out; the caller gathers every rank's handle in rank order (e.g. torch.distributed.all_gather_object)
 * and passes them to tr_gpu_moe_ep_peer_open. Per layer call, every rank in step, all enqueued on `stream`
 * (no host synchronisation; a CUDA graph can hold them):
 *   1. tr_gpu_moe_layer_part(part 0) routes the rank's tokens (sel_id, sel_w outputs);
 *   2. tr_gpu_moe_ep_dispatch writes each (token, slot) row and its expert id straight into its owner's region
 *      (unused slots: id -1), then the owner's arrival flag; d_place[j] = where row j's output comes back;
 *   3. tr_gpu_moe_ep_experts waits for every source's rows, computes them (one fused kernel: the context's
 *      max_tokens must be >= n_ranks x cap, and n_ranks x cap <= 64), writes each output row straight back into
 *      its source's region, then the source's return flag;
 *   4. tr_gpu_moe_ep_peer_combine waits for every owner's rows, then x[t] += the id-ordered mix (and ffn_out).
 * Every wait on another rank is bounded (10 s); a rank that gives up sets the error flag tr_gpu_moe_check
 * reports. 0 or -1. */
#define TRMOE_IPC_HANDLE_BYTES 64
TRMOE_API int tr_gpu_moe_ep_peer_region(tr_gpu_moe *m, int32_t n_ranks, int32_t rank, int64_t cap, void *ipc_handle_out);
TRMOE_API int tr_gpu_moe_ep_peer_open(tr_gpu_moe *m, const void *ipc_handles);
TRMOE_API int tr_gpu_moe_ep_dispatch(tr_gpu_moe *m, const int64_t *d_sel_id, int64_t n_tok, const float *d_normed,
                                     int32_t *d_place, void *stream);
TRMOE_API int tr_gpu_moe_ep_experts(tr_gpu_moe *m, int64_t layer, void *stream);
TRMOE_API int tr_gpu_moe_ep_peer_combine(tr_gpu_moe *m, const float *d_sel_w, const int32_t *d_place, int64_t n_tok,
                                         float *d_x, float *d_ffn_out, void *stream);

/* No counterpart in the reference (its long passes run the same scalar definition): calls of at least min_tokens
 * tokens take the tensor-core road (weights Q8_0, Q4_K or Q6_K; router, top-k and dispatch exact as always; expert
 * products as 3xTF32 tcgen05 GEMMs, within 1e-5 relative of the exact result; combine exact). 0 keeps every call on
 * the exact road. Default 256, or 32 when the down weights are Q4_K (their exact road costs about 74 us a token).
 * Returns 0, or -1 (a non-zero min_tokens on a context without the road). */
TRMOE_API int tr_gpu_moe_set_prefill(tr_gpu_moe *m, int64_t min_tokens);

/* tr_gpu_moe_layer on device memory, enqueued on `stream` (a cudaStream_t; NULL: the context's own
 * stream) and returning without waiting. d_normed and d_x_inout are device pointers. 0, or -1. */
TRMOE_API int tr_gpu_moe_layer_dev(tr_gpu_moe *m, int64_t layer, const float *d_normed, int64_t n_tok, float *d_x_inout,
                         const tr_gpu_moe_outputs *out, void *stream);

/* tr_gpu_moe_ffn on device pointers, enqueued on `stream` (NULL: the context's own), not waited for: d_x_inout
 * normalised and given the layer's output; d_normed_out (optional) receives the normalised rows; out as
 * tr_gpu_moe_layer_dev. */
TRMOE_API int tr_gpu_moe_ffn_dev(tr_gpu_moe *m, int64_t layer, int64_t n_tok, float *d_x_inout, float *d_normed_out,
                                 const tr_gpu_moe_outputs *out, void *stream);

/* One part of tr_gpu_moe_layer_dev: 0 route (router, top-k, dispatch, input preparation), 1 gate/up and
 * SwiGLU, 2 the down input's Q4_K preparation (nothing for another down type), 3 down, combine and residual
 * add: Trochilus's profiler zones ROUTER, EXPERT_GATE_UP, EXPERT_ACT, EXPERT_DOWN + EXPERT_MIX
 * (src/base/prof.h:42-47). Parts 0..3 enqueued in order on one stream with the same arguments are one layer
 * call; `out` is read by the parts that write it (0: logits, sel_id, sel_w, offsets, place; 3: ffn_out).
 * Enqueues only, like tr_gpu_moe_layer_dev; it can be captured in a CUDA graph. 0, or -1. */
TRMOE_API int tr_gpu_moe_layer_part(tr_gpu_moe *m, int64_t layer, int part, const float *d_normed, int64_t n_tok,
                                    float *d_x_inout, const tr_gpu_moe_outputs *out, void *stream);

/* Zone timing, the GPU counterpart of Trochilus's profiler zones (src/base/prof.h:42-47: ROUTER,
 * EXPERT_GATE_UP, EXPERT_ACT, EXPERT_DOWN with EXPERT_MIX): when on, every layer call records CUDA events
 * around its kernels on the stream it runs on. tr_gpu_moe_profile_read waits for the last call and
 * returns, per zone, the summed milliseconds and the calls counted since profiling was switched on:
 * zone 0 router + top-k + dispatch, 1 gate/up + SwiGLU, 2 the down input's Q4_K preparation (0 calls when
 * the down is not Q4_K), 3 down + combine + residual. 0, or -1. */
#define TRMOE_ZONES 4
TRMOE_API int tr_gpu_moe_profile(tr_gpu_moe *m, int on);
TRMOE_API int tr_gpu_moe_profile_read(tr_gpu_moe *m, double *ms, int64_t *calls, int n_zones);

/* Waits for the context's stream and reports whether a kernel gave up on a bounded wait since the last
 * check (the device error flag, then cleared). 0, or -1 with a message. tr_gpu_moe_layer checks it itself. */
TRMOE_API int tr_gpu_moe_check(tr_gpu_moe *m);

/* Timeline of the fused kernel (the counterpart of Trochilus's TR_POOL_TRACE, src/base/threads.h:98-108): when
 * on, every CTA of the fused kernel writes %globaltimer (ns) at its events into 64 slots: 0 start, 1 router or
 * preparation work done, 2 routing seen, 3 copies armed, 4+j gate/up chunk j done (j < 16), 20+j down chunk j's
 * inputs ready, 36+j down chunk j done, 52 end (0: no such event). The one-token kernel: 0 start, 62 logit
 * published, 1 logits held, 60 routed, 8+j warp 0's step j weights in, 24+j its h rows in, 16+j step done, 32+i
 * expert i's h gathered, 6 experts done, 52 end. tr_gpu_moe_trace_read waits for the stream and
 * copies the last call's slots (ctas * 64 values, at most n) to host memory; returns the number of CTAs, or -1. */
TRMOE_API int tr_gpu_moe_trace(tr_gpu_moe *m, int on);
TRMOE_API int tr_gpu_moe_trace_read(tr_gpu_moe *m, uint64_t *slots, int64_t n);

/* How many kernels one tr_gpu_moe_layer_dev call launches for n_tok tokens (without dispatch outputs). */
TRMOE_API int tr_gpu_moe_launches(const tr_gpu_moe *m, int64_t n_tok);

/* The kernel one tr_gpu_moe_layer_dev call of n_tok tokens runs when it is a single kernel: "trx_k_dec1" (the
 * one-token decode kernel; also for calls of up to 64 tokens on its shapes, which launch it once a token),
 * "trx_k_layer" (the fused layer kernel); "" when the call takes several different kernels. */
TRMOE_API const char *tr_gpu_moe_kernel_name(const tr_gpu_moe *m, int64_t n_tok);

/* The message of this thread's last failure ("" if none). */
TRMOE_API const char *trmoe_last_error(void);

/* The architecture the library's device code was built for, as the CUDA runtime reports it for the fused decode
 * kernel on the current device (cudaFuncGetAttributes' binaryVersion: 100 for sm_100a), or -1 with
 * trmoe_last_error() set when there is no device or the code cannot run on it. No counterpart in the reference. */
TRMOE_API int trmoe_kernel_arch(void);

/* ---------------------------------------------------------------------------------------------
 * Decode attention (the rank-3 next step beyond the MoE block): Trochilus's GPU attention backend
 * (src/backend/gpu_attn.h:29-78) on the B200, with the same names, arguments and conventions, so the engine links
 * it in place of src/backend/gpu_attn.c. A session keeps its keys and values in HBM ([layer][head][pos][head_dim]
 * f32); a decode token sends q, k and v and reads back its output, for every head the bits tr_attention_group
 * gives a single query (tr_attention_head, src/kernels/kernels.c:1521-1528). head_dim 128 and one KV head per
 * query head, as the reference supports. */
typedef struct tr_gpu tr_gpu;           /* the device */
typedef struct tr_gpu_attn tr_gpu_attn; /* one session's cache in HBM and its buffers */
#define TRMOE_GPU_WARM_MAX_NS 200000000 /* the longest tr_gpu_attn_warm */
#define TRMOE_GPU_VRAM_RESERVE ((uint64_t)512 << 20) /* HBM a cache must leave free */

/* Replaces: tr_gpu_open (gpu_attn.h:37): the first device of compute capability 10.0 (the library's kernels are
 * built for sm_100a). NULL with a message when there is no driver or no such device. */
TRMOE_API tr_gpu *tr_gpu_open(char *err, size_t err_len);
/* Replaces: tr_gpu_close (gpu_attn.h:38). NULL: nothing. Every session of the device is freed first. */
TRMOE_API void tr_gpu_close(tr_gpu *g);
/* Replaces: tr_gpu_name (gpu_attn.h:40). */
TRMOE_API const char *tr_gpu_name(const tr_gpu *g);
/* Replaces: tr_gpu_attn_create (gpu_attn.h:46-47): a cache of n_ctx positions for every layer and head. NULL with a
 * message when the shape is not supported (head_dim 128) or HBM would keep less than TRMOE_GPU_VRAM_RESERVE free.
 * One session, one thread at a time (the calls make the device current on the calling thread). */
TRMOE_API tr_gpu_attn *tr_gpu_attn_create(tr_gpu *g, int64_t n_layers, int64_t n_head, int64_t head_dim,
                                          int64_t n_ctx, char *err, size_t err_len);
/* Replaces: tr_gpu_attn_free (gpu_attn.h:48). NULL: nothing. */
TRMOE_API void tr_gpu_attn_free(tr_gpu_attn *a);
/* Replaces: tr_gpu_attn_bytes (gpu_attn.h:50): HBM a session of that shape takes. */
TRMOE_API uint64_t tr_gpu_attn_bytes(int64_t n_layers, int64_t n_head, int64_t head_dim, int64_t n_ctx);
/* Replaces: tr_gpu_attn_write (gpu_attn.h:57): positions pos0 .. pos0 + n_tok - 1 of one layer, k and v
 * [n_tok][n_head * head_dim] host rows. Returns when the GPU holds them. 0, or -1 (a range outside the cache). */
TRMOE_API int tr_gpu_attn_write(tr_gpu_attn *a, int64_t layer, int64_t pos0, int64_t n_tok, const float *k,
                                const float *v);
/* Replaces: tr_gpu_attn_decode (gpu_attn.h:65-66): one decode token of one layer at position pos: stores k and v at
 * pos, attends to positions 0 .. pos and writes out [n_head * head_dim], head h the bits
 * tr_attention_head(q + h * head_dim, keys, values, n_head * head_dim, h * head_dim, pos + 1, head_dim, scale, ...)
 * writes. Host rows (pinned or not). 0, or -1 on a CUDA error, a give-up of a bounded wait, or pos outside the
 * cache: the caller then stays on the CPU, whose own cache is whole. */
TRMOE_API int tr_gpu_attn_decode(tr_gpu_attn *a, int64_t layer, int64_t pos, const float *q, const float *k,
                                 const float *v, float scale, float *out);
/* Replaces: tr_gpu_attn_warm (gpu_attn.h:74): keeps one warp of the GPU busy for ns nanoseconds (at most
 * TRMOE_GPU_WARM_MAX_NS) or until the next decode call starts, so that clocks a long idle lowered are up again. 0,
 * or -1. */
TRMOE_API int tr_gpu_attn_warm(tr_gpu_attn *a, uint64_t ns);

/* ---------------------------------------------------------------------------------------------
 * 2. The kernel level (Trochilus src/kernels/kernels.h) */

typedef struct tr_pool tr_pool; /* the reference's thread pool: accepted and ignored */

/* Trochilus's tr_mat (src/kernels/kernels.h:69-76): `rows` rows of `cols` elements of `type`, ggml
 * layout. The type is a ggml type number (an enum in the reference, an int here: same size). */
typedef struct {
    int32_t type;
    int64_t rows;
    int64_t cols;
    const void *data;
} tr_mat;

/* Replaces: tr_matmul (src/kernels/kernels.h:239). y[t*rows + r] = row r of w . x[t*cols ..]. */
TRMOE_API void tr_matmul(tr_pool *pool, const tr_mat *w, const float *x, int64_t n_tokens, float *y);
/* Replaces: tr_matmul_grouped (src/kernels/kernels.h:244-245). Group g holds input rows
 * [offsets[g], offsets[g+1]) and multiplies them by w[g]; empty groups skipped. */
TRMOE_API void tr_matmul_grouped(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups, const float *x,
                       float *y);
/* Replaces: tr_matmul_grouped_s (src/kernels/kernels.h:277-278); the scratch argument is ignored (the
 * GPU keeps its own), the result is tr_matmul_grouped's. */
TRMOE_API void tr_matmul_grouped_s(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups, const float *x,
                         float *y, const void *s);
/* Replaces: tr_softmax (src/kernels/kernels.h:342): in place over n logits. */
TRMOE_API void tr_softmax(float *x, int64_t n);
/* Replaces: tr_swiglu (src/kernels/kernels.h:345): x[i] = silu(x[i]) * y[i]. */
TRMOE_API void tr_swiglu(tr_pool *pool, float *x, const float *y, int64_t n);
/* Replaces: tr_matmul_s (src/kernels/kernels.h:279): tr_matmul's result; the scratch argument is ignored. */
TRMOE_API void tr_matmul_s(tr_pool *pool, const tr_mat *w, const float *x, int64_t n_tokens, float *y, const void *s);

/* Q4_K's prepared road (src/kernels/kernels.h:280-300, 346-350). The engine prepares a pass's input rows once into
 * its own buffer, one slot of tr_q4x_bytes(cols) bytes a row, and every Q4_K matmul of the pass reads them, a
 * group's input row p from slot map[p]. In this library a slot holds the row's floats at its start; the GPU prepares
 * the integer digits inside each matmul from those floats, so every output is the reference road's (which equals
 * tr_matmul_grouped_s's bit for bit, kernels.h:286-292). The slots' format is the library's own: the engine must take
 * these six functions together (tr_q4x_road, tr_q4x_prepare, tr_matmul_q4x_prepared, tr_matmul_q4x_prepared_n,
 * tr_swiglu_prepare and tr_matmul_s), never mix them with the CPU's. Pool and scratch are not consulted. */
/* Replaces: tr_q4x_bytes (src/kernels/kernels.h:90): the bytes of one slot, the reference's formula. */
TRMOE_API size_t tr_q4x_bytes(int64_t n);
/* Replaces: tr_q4x_road (src/kernels/kernels.h:289): 1 when w[0] is Q4_K, its rows a multiple of 16 and its
 * columns a positive multiple of 256 (the calls the library's Q4_K road takes), else 0. */
TRMOE_API int tr_q4x_road(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups, const void *s);
/* Replaces: tr_q4x_prepare (src/kernels/kernels.h:288): rows 0..n-1 of x (cols floats each) into xq, row r's
 * floats at byte r * tr_q4x_bytes(cols). A host copy: the GPU is not involved. */
TRMOE_API void tr_q4x_prepare(tr_pool *pool, const float *x, int64_t n, int64_t cols, void *xq);
/* Replaces: tr_matmul_q4x_prepared (src/kernels/kernels.h:290-291): y[p*rows + r] = row r of w[g(p)] . the row in
 * slot map[p] of xq (map NULL: slot p). 1 when done (an empty call included); 0, y untouched, when tr_q4x_road
 * refuses w. A GPU failure prints `trmoe: tr_matmul_q4x_prepared failed: <reason>`, fills y with NaN and returns 1. */
TRMOE_API int tr_matmul_q4x_prepared(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups,
                                     const void *xq, const int64_t *map, float *y, const void *s);
/* Replaces: tr_matmul_q4x_prepared_n (src/kernels/kernels.h:298-299): the same for n_w (1..TRMOE_Q4X_MATS) weights of
 * one shape on the same groups and slots, y[m] from w[m]; the rows go to the GPU and are prepared once for all of
 * them. 0, every y untouched, when n_w is out of range, a weight is refused or the shapes differ. */
#define TRMOE_Q4X_MATS 3
TRMOE_API int tr_matmul_q4x_prepared_n(tr_pool *pool, const tr_mat *const *w, int n_w, const int64_t *offsets,
                                       int64_t n_groups, const void *xq, const int64_t *map, float *const *y,
                                       const void *s);
/* Replaces: tr_q4x_fused_calls (src/kernels/kernels.h:300): tr_matmul_q4x_prepared_n's calls of n_w > 1 so far. */
TRMOE_API uint64_t tr_q4x_fused_calls(void);
/* Replaces: tr_swiglu_prepare (src/kernels/kernels.h:350): tr_swiglu over n_rows rows of n, then row r's floats into
 * xq at byte r * tr_q4x_bytes(n) (the down's slots). */
TRMOE_API void tr_swiglu_prepare(tr_pool *pool, float *x, const float *y, int64_t n_rows, int64_t n, void *xq);

/* No counterpart in the reference (it has no GPU matmul API). y[t*rows + r] = row r of a Q4_K matrix . x[t*cols ..],
 * bit for bit tr_matmul's result, for callers that cannot allocate device memory: a process whose HBM is all held
 * by another allocator (a serving engine that reserves it at start-up), or code that must not call cudaMalloc /
 * cudaFree because they can synchronise the device behind other streams' backs.
 * Every pointer is caller-owned DEVICE memory on the calling thread's current device: d_w = rows GGUF Q4_K rows
 * (144 B per 256 columns), d_x = n_tokens x cols f32, d_y = n_tokens x rows f32; cols a multiple of 256; d_w and
 * d_x 16-byte aligned. The prepared inputs go to a fixed scratch array inside the library, of
 * TRMOE_NOALLOC_SCRATCH_BYTES on every GPU that loads it, held until the process exits. A call needs 256 bytes of
 * it plus, per token, cols * 4 + cols / 4 + cols / 32 bytes (each part rounded up to 256), so 2048 columns fit
 * 478 tokens; a larger call is rejected with an error. A successful call allocates nothing, host or device.
 * The first call on a device looks up the scratch's device address (cudaGetSymbolAddress) and keeps it: make
 * that first call before any stream capture. Under lazy module loading (CUDA_MODULE_LOADING=LAZY, the default of
 * recent CUDA runtimes) that first call, or the first launch of a kernel, may also load the library's device code,
 * which the driver may back with device memory of its own; the calls after it allocate nothing. Every call shares the one scratch array and leaves its contents
 * there: calls that may overlap on the GPU (different streams, or different host threads on one device) race,
 * and the caller must serialise them. Asynchronous on `stream` (NULL: the default stream); returns 0, or -1 with
 * trmoe_last_error() set. */
#define TRMOE_NOALLOC_SCRATCH_BYTES 4194304
TRMOE_API int tr_matmul_q4k_noalloc(const void *d_w, int64_t rows, int64_t cols, const float *d_x, int64_t n_tokens,
                                    float *d_y, void *stream);

/* Drops every weight the kernel level uploaded (the next call uploads again). */
TRMOE_API void trmoe_kernel_cache_clear(void);

#ifdef __cplusplus
}
#endif

#endif
