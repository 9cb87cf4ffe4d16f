/*
 * nf_moe.h -- C ABI of the B200 (sm_100a) NVFP4 routed-expert MoE layer.
 *
 * This library replaces the CPU path of GLM-5.3-Flash's MoE feed-forward in
 * alan70435-vibe/Ninfer_Nvfp4_Glm-5.3_Flash_2x_DgxSpark.  Every entry point
 * cites the reference interface it stands in for (file:line inside that
 * project).  The reference has no plugin or FFI layer: its MoE path is the
 * private member TextModel::moe, so the entry points below are the ones a
 * maintainer binds from the reference's C++ host (a handle per MoE layer,
 * bound from the Store by checkpoint name, called from TextModel::moe).
 * Conventions:
 *   - every call returns an int status (NF_OK == 0); no exception or C++
 *     type crosses the ABI; nf_moe_last_error() gives the message, worded
 *     like the reference's std::runtime_error messages;
 *   - pointers named *_dev are device pointers on the handle's device,
 *     *_host are host pointers; sizes are element counts;
 *   - bind calls copy host data into device memory owned by the handle (the
 *     caller's checkpoint mmaps only need to live during the call) and
 *     validate before any device write;
 *   - one handle per (device, stream); a handle is not thread-safe;
 *   - nf_moe_forward allocates nothing: every workspace is sized at create
 *     time from nf_moe_desc.max_tokens.
 */
#ifndef NF_MOE_H
#define NF_MOE_H

#include <stdint.h>

#if defined(__GNUC__)
#define NF_API __attribute__((visibility("default")))
#else
#define NF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum {
    NF_OK = 0,
    NF_ERR_INVALID = 1,     /* bad argument (null pointer, out-of-range id) */
    NF_ERR_SHAPE = 2,       /* "NVFP4 shape <name>" / "BF16 linear layout <name>" */
    NF_ERR_LAYOUT = 3,      /* "NVFP4 layout <name>" */
    NF_ERR_SCALE = 4,       /* "NVFP4 input scale", bad block / global scale */
    NF_ERR_STATE = 5,       /* weights missing, not finalized, already finalized */
    NF_ERR_CUDA = 6,        /* a CUDA runtime call failed */
    NF_ERR_TIMEOUT = 7,     /* a device-side bounded wait gave up */
    NF_ERR_UNSUPPORTED = 8, /* a descriptor this build does not implement */
    NF_ERR_NOMEM = 9,       /* device allocation failed at create/bind time */
    NF_ERR_CAPACITY = 10    /* tokens > max_tokens */
};

/* NVFP4 projection ids (parameter_schema add_nvfp4 prefixes,
 * src/parameter_schema.cpp:93-95). */
enum { NF_PROJ_GATE = 0, NF_PROJ_UP = 1, NF_PROJ_DOWN = 2 };

/* BF16 tensor ids (src/parameter_schema.cpp:76-82 and the BF16 MTP experts
 * :87-91). */
enum {
    NF_BF16_ROUTER = 0,      /* mlp.gate.weight                  [E, H]  */
    NF_BF16_SHARED_GATE = 1, /* mlp.shared_experts.gate_proj     [Is, H] */
    NF_BF16_SHARED_UP = 2,   /* mlp.shared_experts.up_proj       [Is, H] */
    NF_BF16_SHARED_DOWN = 3, /* mlp.shared_experts.down_proj     [H, Is] */
    NF_BF16_EXPERT_GATE = 4, /* mlp.experts.<e>.gate_proj.weight [I, H]  (layer-45 BF16 experts) */
    NF_BF16_EXPERT_UP = 5,   /* mlp.experts.<e>.up_proj.weight   [I, H]  */
    NF_BF16_EXPERT_DOWN = 6  /* mlp.experts.<e>.down_proj.weight [H, I]  */
};

/* F32 tensor ids. */
enum { NF_F32_ROUTER_BIAS = 0 /* mlp.gate.e_score_correction_bias [E] (src/parameter_schema.cpp:78-79) */ };

/* Routed expert storage. */
enum { NF_EXPERTS_NVFP4 = 0, NF_EXPERTS_BF16 = 1 };

/* Layer descriptor.  Filled from ModelSpec (include/ninfer_glm53/model_spec.hpp:
 * hidden_size, routed_experts, experts_per_token, moe_intermediate_size,
 * routed_scaling_factor, swiglu_limit) or from a synthetic configuration.
 * Limits of this build: hidden % 256 == 0, inter % 128 == 0,
 * shared_inter % 128 == 0 (or 0 for no shared expert), 1 <= top_k <= 32,
 * top_k <= experts <= 1024. */
typedef struct nf_moe_desc {
    int32_t hidden;         /* H */
    int32_t experts;        /* E, routed experts (global, before EP sharding) */
    int32_t top_k;          /* experts per token */
    int32_t inter;          /* I, routed expert intermediate size */
    int32_t shared_inter;   /* shared expert intermediate size, 0 = none */
    int32_t n_group;        /* group-limited routing: expert groups (1 = off) */
    int32_t topk_group;     /* groups kept when n_group > 1 */
    int32_t normalize;      /* renormalise top-k weights (router_select normalize) */
    float routed_scaling;   /* routed_scaling_factor */
    float swiglu_limit;     /* swiglu_limit */
    int32_t expert_kind;    /* NF_EXPERTS_NVFP4 or NF_EXPERTS_BF16 */
    int32_t max_tokens;     /* workspace capacity per forward */
} nf_moe_desc;

typedef struct nf_moe nf_moe;

/* Creates a handle on `device` (which becomes current for the call) and
 * allocates the device weights and workspace.  Replaces TextModel's
 * construction of the MoE state (src/text_forward.cpp:580-623). */
NF_API int nf_moe_create(const nf_moe_desc* desc, int device, nf_moe** out);
NF_API void nf_moe_destroy(nf_moe* handle);
/* Message of the handle's last failure ("" when none).  With a NULL handle,
 * the message of the last failed nf_moe_create on this thread. */
NF_API const char* nf_moe_last_error(const nf_moe* handle);
NF_API const char* nf_status_string(int status);

/* Binds one NVFP4 expert projection: packed U8 [rows, cols/2] (low nibble =
 * even column), F8_E4M3 block scales [rows, cols/16], rank-0 F32
 * weight_scale_2 and input_scale, all in checkpoint order.  Validates what
 * linear_nvfp4 (src/text_forward.cpp:832-843) and Nvfp4MatrixView
 * (src/nvfp4_decode.cpp:56-79) validate: rows/cols match the descriptor
 * ("NVFP4 shape"), cols % 16, finite positive input_scale ("NVFP4 input
 * scale"), finite weight_scale_2 >= FLT_MIN, block scales finite and
 * non-negative.  gate and up of one expert must carry the same input_scale
 * in this build (ModelOpt calibrates both on the same input). */
NF_API int nf_moe_bind_nvfp4(nf_moe* handle, int expert, int proj, const uint8_t* packed_host, const uint8_t* scales_host,
                      float weight_scale_2, float input_scale, int64_t rows, int64_t cols);
/* Binds a BF16 matrix (see the NF_BF16_* ids; `expert` is ignored for the
 * router and shared tensors).  Checks the shape like linear_bf16
 * (src/text_forward.cpp:821-825, "BF16 linear layout <name>"). */
NF_API int nf_moe_bind_bf16(nf_moe* handle, int which, int expert, const uint16_t* data_host, int64_t rows, int64_t cols);
/* Binds an F32 vector (router correction bias, Store::load
 * src/text_forward.cpp:478-491, "vector length mismatch"). */
NF_API int nf_moe_bind_f32(nf_moe* handle, int which, const float* data_host, int64_t n);
/* Checks that every tensor the descriptor needs is bound and builds the
 * device layouts (block-scale atoms, gate/up interleave).  Required once
 * before the first forward. */
NF_API int nf_moe_finalize(nf_moe* handle);

/* The MoE layer for `tokens` tokens, enqueued on `stream` (cudaStream_t,
 * NULL = legacy default stream).  Replaces TextModel::moe
 * (src/text_forward.cpp:924-963) stepped over each token, plus the hc = 1
 * residual form of mhc_combine (src/text_forward.cpp:906, 1646-1657):
 *   x_dev        BF16 [tokens, H] (the rmsnorm_stash output, BF16-valued)
 *   residual_dev F32 [tokens, H] or NULL (NULL: y is the FFN branch alone)
 *   y_dev        F32 [tokens, H]
 *   (x_dev, residual_dev and y_dev 16-byte aligned, else NF_ERR_LAYOUT)
 *   topk_idx_dev INT32 [tokens, top_k] or NULL (router_select indices)
 *   topk_w_dev   F32 [tokens, top_k] or NULL (router_select weights)
 * With tokens == 0 nothing is read or written, so x_dev and y_dev may be
 * NULL (an expert-parallel rank without tokens still makes the call).
 * Asynchronous: a device-side failure (bounded wait timeout) is reported by
 * the next call that synchronises (nf_moe_sync or nf_moe_forward_host). */
NF_API int nf_moe_forward(nf_moe* handle, const uint16_t* x_dev, const float* residual_dev, int tokens, float* y_dev,
                   int32_t* topk_idx_dev, float* topk_w_dev, void* stream);
/* Host-buffer form with the reference's own contract (fp32 in, fp32 out;
 * moe(prefix, x, y) src/text_forward.cpp:924): copies x (BF16-valued F32,
 * rounded to BF16 on the device) and residual to the device, runs the layer
 * on the handle's internal stream, copies y (and the routes when the
 * pointers are not NULL) back and synchronises.  In graph mode, with every
 * host buffer page-locked, the copies and the layer replay as one graph per
 * distinct set of buffers. */
NF_API int nf_moe_forward_host(nf_moe* handle, const float* x_host, const float* residual_host, int tokens, float* y_host,
                        int32_t* topk_idx_host, float* topk_w_host);
/* Graph mode (off by default): nf_moe_forward captures its launches for each
 * distinct (x, residual, y, idx, w, tokens, stream) into a CUDA graph on
 * first use and replays the graph afterwards (the 16 most recent argument
 * sets are kept).  Needs a non-NULL stream; forwards with per-stage
 * profiling on, on the NULL stream, or issued while the caller is capturing
 * run the kernels directly. */
NF_API int nf_moe_set_graph_mode(nf_moe* handle, int enable);
/* The grouped NVFP4 expert GEMMs of batches with at least 256 routed rows per
 * expert on average (prefill): NF_GEMM_ONE_SM (default) runs 128 x 256 tiles
 * with 256-K stages on each SM; NF_GEMM_WIDE_STAGES the same tiles with 512-K
 * stages (half the TMA copies per MMA, two stages deep); NF_GEMM_CTA_PAIR
 * 256 x 256 tiles on pairs of SMs (tcgen05 cta_group::2) with the activation
 * rows resident.  Smaller batches always take the first.  The results agree
 * within the layer tolerance (the same K order per output). */
enum { NF_GEMM_ONE_SM = 0, NF_GEMM_WIDE_STAGES = 1, NF_GEMM_CTA_PAIR = 2 };
NF_API int nf_moe_set_expert_gemm(nf_moe* handle, int mode);
/* Waits for the handle's work on `stream` and reports a device-side error. */
NF_API int nf_moe_sync(nf_moe* handle, void* stream);

/* ---- stage-level entry points (parity tests and profiling) ---------------
 * Router only: logits (optional, F32 [tokens, E]), indices and weights.
 * gemv_bf16 + router_select (src/text_forward.cpp:926-931, 497-508,
 * 1447-1471), bit-exact. */
NF_API int nf_moe_route(nf_moe* handle, const uint16_t* x_dev, int tokens, float* logits_dev, int32_t* topk_idx_dev,
                 float* topk_w_dev, void* stream);

/* Internal buffers of the last forward, for parity tests.  Returns the
 * device pointer and its size in bytes. */
enum {
    NF_DBG_COUNTS = 0,      /* INT32 [E]          tokens routed to each expert          */
    NF_DBG_SEG_OFFSET = 1,  /* INT32 [E + 1]      first permuted row of each expert      */
    NF_DBG_PAIR_ROW = 2,    /* INT32 [T, top_k]   permuted row of each (token, pick)     */
    NF_DBG_ROW_TOKEN = 3,   /* INT32 [rows]       token of each permuted row, -1 = pad   */
    NF_DBG_ACT_CODES = 4,   /* U8    [rows, H/2]  E2M1 codes of the gate/up input        */
    NF_DBG_ACT_SF = 5,      /* U8    E4M3 block scales of the gate/up input (atom layout) */
    NF_DBG_H_CODES = 6,     /* U8    [rows, I/2]  E2M1 codes of the down input           */
    NF_DBG_H_SF = 7,        /* U8    E4M3 block scales of the down input (atom layout)   */
    NF_DBG_DOWN = 8,        /* BF16 [rows, H] (NVFP4) or F32 (BF16 experts): down output */
    NF_DBG_SHARED = 9,      /* F32   [T, H]       shared expert output                   */
    NF_DBG_ROWS = 10,       /* INT32 [1]          permuted rows in use (incl. padding)   */
    NF_DBG_LOGITS = 11,     /* F32   [T, E]       router logits: exact (full router), or the tensor-core
                                                  approximations the screened router bounds */
    NF_DBG_SCREEN_COUNT = 12 /* INT32 [T]         screened router: exact chains per token, -1 = all E */
};
NF_API int nf_moe_debug_tensor(nf_moe* handle, int which, void** dev_ptr, int64_t* bytes);
/* Copies the first `bytes` bytes of a debug tensor to host memory
 * (synchronous; waits for the handle's device work first). */
NF_API int nf_moe_debug_read(nf_moe* handle, int which, void* host_dst, int64_t bytes);

/* Per-stage timing with CUDA events recorded on the forward's stream.
 * enable != 0 starts recording (and clears the totals); every forward then
 * adds the device time of each stage.  nf_moe_stage_times synchronises and
 * returns the accumulated milliseconds per stage (NF_STAGE_COUNT values)
 * and the number of forwards recorded. */
enum {
    NF_STAGE_ROUTER = 0,
    NF_STAGE_PERMUTE = 1,
    NF_STAGE_GATE_UP = 2,
    NF_STAGE_DOWN = 3,
    NF_STAGE_SHARED = 4,
    NF_STAGE_COMBINE = 5,
    NF_STAGE_COUNT = 6
};
NF_API int nf_moe_profile(nf_moe* handle, int enable);
NF_API int nf_moe_stage_times(nf_moe* handle, float* ms_out, int* forwards);

/* NVFP4 dequantisation: out[r, c] = e2m1 * e4m3(scale) * global_scale with
 * one rounding (Nvfp4MatrixView::at, src/nvfp4_decode.cpp:88-97), after the
 * view constructor's validation (src/nvfp4_decode.cpp:56-79), which reads the
 * scales back to the host.  Synchronous. */
NF_API int nf_nvfp4_dequantize(const uint8_t* packed_dev, const uint8_t* scales_dev, float global_scale, int64_t rows,
                        int64_t cols, float* out_dev, void* stream);
/* NVFP4 activation quantiser (quant_dequant_nvfp4_activation,
 * src/text_forward.cpp:527-550) on F32 rows: codes [rows, cols/2], E4M3
 * scales [rows, cols/16] in plain row-major order, optional fake-quant
 * values [rows, cols] (e2m1 * scale, the reference's output vector). */
NF_API int nf_nvfp4_quantize(const float* x_dev, int64_t rows, int64_t cols, float input_scale, uint8_t* codes_dev,
                      uint8_t* scales_dev, float* fake_dev, void* stream);
/* Sigmoid exactly as the reference computes it (src/text_forward.cpp:42-49,
 * libm expf), element-wise over n floats. */
NF_API int nf_sigmoid_ref(const float* x_dev, int64_t n, float* y_dev, void* stream);
/* Checks, on the current device and over every 32-bit pattern, that the
 * hardware E2M1, E4M3 and BF16 conversions the kernels use agree with the
 * reference's encoders (cast_to_e2m1, src/text_forward.cpp:510-522, after
 * the +-6 clamp; f32_to_e4m3, :60-85, on [2^-6, inf) after the 448 clamp;
 * f32_to_bf16, :87-95, on every non-NaN input).  Returns the mismatch
 * counts (all 0 on a correct build).  Synchronous. */
NF_API int nf_format_selfcheck(int64_t* e2m1_mismatches, int64_t* e4m3_mismatches, int64_t* bf16_mismatches);

/* ---- dense NVFP4 MLP (layers 0-2) ------------------------------------------
 * Creates a handle for the dense feed-forward of the first layers,
 * TextModel::dense_mlp (src/text_forward.cpp:909-915), selected by feed()
 * for FfnKind::kDense (src/text_forward.cpp:903): NVFP4 gate and up linears
 * (linear_nvfp4 :832-856, outputs rounded to BF16), swiglu_clamp_bf16
 * (:99-106: BF16 after the clamps, after SiLU and after the product), NVFP4
 * down linear.  Limits: hidden % 256 == 0, inter % 128 == 0.
 * The handle is an nf_moe handle with one expert and no router:
 *   - bind with nf_moe_bind_nvfp4(handle, 0, NF_PROJ_GATE / UP / DOWN, ...)
 *     the checkpoint's mlp.gate_proj / up_proj / down_proj tensors
 *     (parameter_schema's dense layers, src/parameter_schema.cpp:187-191);
 *     gate is [inter, hidden], down [hidden, inter]; messages name
 *     "mlp.<proj>";
 *   - nf_moe_finalize, nf_moe_forward / nf_moe_forward_host (topk pointers
 *     must be NULL), nf_moe_set_graph_mode, nf_moe_profile and
 *     nf_moe_destroy work as for a MoE layer; y = down + residual (or down
 *     alone when residual is NULL), the hc = 1 form of mhc_combine (:906). */
NF_API int nf_moe_create_dense(int32_t hidden, int32_t inter, float swiglu_limit, int32_t max_tokens, int device,
                               nf_moe** out);

/* ---- expert parallelism ----------------------------------------------------
 * The layer sharded by experts over `world` GPUs of one node (1 <= world <= 8,
 * experts % world == 0), one handle per rank and GPU; the reference runs one
 * process per GPU with a TP split of the dense projections
 * (src/text_forward.cpp:242-256, src/execution_plan.cpp:69-70) and has no
 * expert parallelism.  Rank r owns experts [r E/world, (r+1) E/world); the
 * router and the shared expert are replicated; every rank passes its own
 * tokens (max_tokens per rank).  The host of rank 0 makes a group id with
 * nf_ep_unique_id and hands it to every rank (by any means); each rank
 * creates its handle with it.  Binding: pass every expert (global ids); a
 * rank keeps the ones it owns and skips the others.  Every rank must call
 * nf_moe_forward (or nf_moe_forward_host) for each step, also with tokens ==
 * 0: the forward exchanges rows with the other ranks (NCCL point-to-point,
 * loaded from libnccl.so.2 at the first EP handle, or NVLink peer memory:
 * see nf_moe_ep_transport).
 * Results are bit-identical to one GPU holding every expert.
 * Create is collective: a rank whose own part fails (an allocation, its
 * experts handle) still joins the communicator and the first set-up
 * exchange and reports its status there, so every rank's create returns
 * that status ("expert-parallel set-up failed on rank p (...)") instead of
 * waiting for the failed rank.  Only a failure of the rank's router and
 * shared-expert part, or of the exchanges' small staging buffer, returns
 * before the communicator exists. */
#define NF_EP_ID_BYTES 128
NF_API int nf_ep_unique_id(uint8_t* group_id_out, int len);
/* Expert parallelism with replicated hot experts: every rank also holds
 * the experts listed in `replicas` (ids in [0, experts), no duplicates; the
 * same list on every rank), and a pick of a replicated expert is computed on
 * the rank whose token made it, with no exchange -- the skew of a few hot
 * experts spreads over the ranks with the tokens.  The outputs stay
 * identical to one GPU bit for bit (rows are independent).  Binding every
 * expert on every rank binds the replicas too.  n_replicas = 0 is
 * nf_moe_create_ep. */
NF_API int nf_moe_create_ep_replicated(const nf_moe_desc* desc, int device, int rank, int world,
                                       const uint8_t* group_id, int id_len, const int32_t* replicas, int n_replicas,
                                       nf_moe** out);
NF_API int nf_moe_create_ep(const nf_moe_desc* desc, int device, int rank, int world, const uint8_t* group_id,
                            int id_len, nf_moe** out);
/* The exchange an EP handle uses (the choice is made collectively at
 * create): NF_EP_NVLINK -- every rank maps every other rank's receive
 * "mailbox" with CUDA IPC and rows and outputs cross NVLink by direct stores
 * with bounded-wait epoch flags, no host synchronisation, so EP forwards run
 * in graph mode too; NF_EP_NCCL -- NCCL point-to-point with one host
 * synchronisation for the row counts.  The environment variable
 * NF_EP_TRANSPORT=nvlink or =nccl chooses (NVLink when unset); NVLink falls
 * back to NCCL when some rank cannot map a mailbox.  NF_EP_NONE for a
 * one-GPU handle.  Over NVLink a rank writes into its peers' mailboxes, so
 * destroy the handles of a group only after every rank's last forward has
 * completed (for example after a host barrier). */
enum { NF_EP_NONE = 0, NF_EP_NCCL = 1, NF_EP_NVLINK = 2 };
NF_API int nf_moe_ep_transport(const nf_moe* handle);

/* ---- tensor-parallel BF16 linears ------------------------------------------
 * The reference splits every BF16 projection by output rows over its two
 * ranks and swaps the halves over a socket: apply_rows
 * (src/text_forward.cpp:803-819) runs gemv_bf16 (:497-508) on rank r's rows,
 * gather_rows (:242-256) gives every rank the whole vector; linear_bf16
 * (:821-830) and the lm_head (:656-667, lm_head_logits :760-767) use it, at
 * the ExecutionPlan's collective boundaries (src/execution_plan.cpp:66-70).
 * A group of `world` GPUs of one node (1-8, one handle per rank and GPU)
 * replaces both steps: each rank computes its rows
 * [rank rows / world, (rank + 1) rows / world) -- for world = 2 the
 * reference's halves -- with gemv_bf16's exact arithmetic and stores them
 * into every rank's gather buffer over NVLink (CUDA IPC, bounded-wait epoch
 * flags), or NCCL point-to-point when the ranks cannot map each other's
 * buffers (NF_TP_TRANSPORT=nccl forces it).  Results are bit-identical to
 * gemv_bf16 over all rows on one rank, whatever the world size. */
typedef struct nf_tp nf_tp;
/* The row block [*row0, *row1) rank `rank` of `world` computes. */
NF_API int nf_tp_split(int64_t rows, int rank, int world, int64_t* row0, int64_t* row1);
/* Creates rank `rank`'s handle on `device` (collective for world > 1: every
 * rank calls it with the same group id from nf_ep_unique_id; world = 1 needs
 * no id).  The handle holds two gather buffers of max_tokens x max_rows F32. */
NF_API int nf_tp_create(int device, int rank, int world, const uint8_t* group_id, int id_len, int max_tokens,
                        int64_t max_rows, nf_tp** out);
NF_API void nf_tp_destroy(nf_tp* handle);
/* Message of the handle's last failure; NULL handle: the last failed create
 * on this thread. */
NF_API const char* nf_tp_last_error(const nf_tp* handle);
/* NF_EP_NONE (world 1), NF_EP_NVLINK or NF_EP_NCCL. */
NF_API int nf_tp_transport(const nf_tp* handle);
/* linear_bf16 over `tokens` tokens (every rank makes the call, in the same
 * order, also with tokens == 0):
 *   w_dev  BF16 [row1 - row0, cols]: this rank's rows of the [rows, cols]
 *          weight (nf_tp_split), 8-byte aligned, cols % 4 == 0
 *   x_dev  F32 [tokens, cols], the same on every rank, 16-byte aligned
 *   y_dev  F32 [tokens, rows] or NULL: the whole output on every rank (it
 *          also stays in the handle until the next call; nf_tp_argmax reads
 *          it there).
 * Enqueued on `stream`; results of a call are valid until the handle's next
 * call, which must be enqueued on the same stream.  A peer that never takes
 * part makes the bounded waits give up: nf_tp_sync then reports
 * NF_ERR_TIMEOUT and the group must be recreated. */
NF_API int nf_tp_linear_bf16(nf_tp* handle, const uint16_t* w_dev, int64_t rows, int64_t cols, const float* x_dev,
                             int tokens, float* y_dev, void* stream);
/* The reference's greedy pick over the last call's output (TextModel::argmax,
 * src/text_forward.cpp:668-681): per token the lowest row with the greatest
 * value; NaN never wins, a NaN in row 0 is kept.  idx_dev INT32 [tokens]. */
NF_API int nf_tp_argmax(nf_tp* handle, int tokens, int64_t rows, int32_t* idx_dev, void* stream);
/* Device address of the last call's [tokens, rows] output inside the handle
 * (synchronous: reads the device's call counter). */
NF_API int nf_tp_result(nf_tp* handle, const float** out_dev);
/* Waits for `stream` and reports a bounded wait that gave up. */
NF_API int nf_tp_sync(nf_tp* handle, void* stream);

/* ---- decoder stack (greedy decode) ------------------------------------------
 * The reference's token step, TextModel::step + argmax
 * (src/text_forward.cpp:625-698), over a synthetic decoder of the benchmark's
 * shape: embedding (embed_row :753), per layer an attention block and the
 * feed-forward that feed() selects (:892-907: the dense NVFP4 MLP :909-915,
 * the NVFP4 MoE :924-963, or BF16 routed experts for the last layers), the
 * final norm (:652-654) and the greedy token over the lm_head (:656-698).
 * The attention block is BF16 GQA with per-head q/k RMSNorm and RoPE, the
 * math of the reference's only GQA attention, draft_attention
 * (:1216-1289): a = rmsnorm(x) (BF16), q/k/v = a . W^T, q and k normed
 * (eps 1e-5) and rotated at the token's position, softmax(q.k / sqrt(128))
 * over the sequence's cache, o = mix . Wo^T, h = x + o; the FFN input is
 * rmsnorm_stash(h) (:267-276) and the layer output h + ffn.  One new token
 * per sequence per step; the caches are BF16 [seq][kv_head][position][128].
 * Limits: head_dim 128, q_heads = 8 kv_heads, hidden % 256 == 0. */
typedef struct nf_stack_desc {
    int32_t vocab;              /* vocabulary (embedding and lm_head rows) */
    int32_t hidden;             /* H */
    int32_t layers;             /* decoder layers */
    int32_t dense_layers;       /* the first layers: dense NVFP4 MLP */
    int32_t bf16_expert_layers; /* the last layers: MoE with BF16 routed experts */
    int32_t dense_inter;        /* dense MLP intermediate size */
    nf_moe_desc moe;            /* the MoE layers (hidden and max_tokens are taken from the stack) */
    int32_t q_heads, kv_heads, head_dim;
    float rope_theta;           /* RoPE base (rope_heads: 10000) */
    float norm_eps;             /* input / post-attention / final RMSNorm epsilon */
    int32_t max_batch;          /* sequences per step */
    int32_t max_context;        /* cache positions per sequence */
} nf_stack_desc;
typedef struct nf_stack nf_stack;
/* Tensor ids of nf_stack_bind_bf16 / _f32 (names of a layer's tensors in the
 * stack's own checkpoint convention: layers.<l>.self_attn.{q,k,v,o}_proj,
 * .input_layernorm, .post_attention_layernorm, .self_attn.{q,k}_norm). */
enum {
    NF_STACK_EMBED = 0,      /* BF16 [vocab, H] */
    NF_STACK_LM_HEAD = 1,    /* BF16 [vocab, H] */
    NF_STACK_Q_PROJ = 2,     /* BF16 [q_heads 128, H]  (per layer) */
    NF_STACK_K_PROJ = 3,     /* BF16 [kv_heads 128, H] */
    NF_STACK_V_PROJ = 4,     /* BF16 [kv_heads 128, H] */
    NF_STACK_O_PROJ = 5,     /* BF16 [H, q_heads 128]  */
    NF_STACK_ATTN_NORM = 6,  /* F32 [H] input_layernorm */
    NF_STACK_FFN_NORM = 7,   /* F32 [H] post_attention_layernorm */
    NF_STACK_Q_NORM = 8,     /* F32 [128] */
    NF_STACK_K_NORM = 9,     /* F32 [128] */
    NF_STACK_FINAL_NORM = 10 /* F32 [H] */
};
NF_API int nf_stack_create(const nf_stack_desc* desc, int device, nf_stack** out);
NF_API void nf_stack_destroy(nf_stack* stack);
NF_API const char* nf_stack_last_error(const nf_stack* stack);
/* The feed-forward handle of a layer: bind its weights with nf_moe_bind_*
 * and nf_moe_finalize (a dense handle for the first dense_layers). */
NF_API nf_moe* nf_stack_layer_ffn(nf_stack* stack, int layer);
NF_API int nf_stack_bind_bf16(nf_stack* stack, int which, int layer, const uint16_t* data_host, int64_t rows,
                              int64_t cols);
NF_API int nf_stack_bind_f32(nf_stack* stack, int which, int layer, const float* data_host, int64_t n);
NF_API int nf_stack_finalize(nf_stack* stack);
/* Device pointers of a layer's K and V caches, BF16 [max_batch][kv_heads]
 * [max_context][128] (post-norm, post-RoPE keys), e.g. to load a history. */
NF_API int nf_stack_kv_cache(nf_stack* stack, int layer, uint16_t** k_dev, uint16_t** v_dev);
/* Copies a layer's whole K and V caches from host memory (the layout above,
 * max_batch x kv_heads x max_context x 128 BF16 each): a loaded history or
 * prefix.  Synchronous. */
NF_API int nf_stack_load_kv(nf_stack* stack, int layer, const uint16_t* k_host, const uint16_t* v_host);
/* Fills every layer's caches on the device with deterministic pseudo-random
 * BF16 values in (-1, 1) derived from `seed`: a stand-in history for timing
 * long contexts.  Synchronous. */
NF_API int nf_stack_fill_kv(nf_stack* stack, uint64_t seed);
/* One greedy decode step for `batch` sequences: sequence i takes token
 * tokens_dev[i] at position positions_dev[i] (keys 0 .. position attended;
 * the new key and value are written at that position), and next_dev[i]
 * receives its greedy token.  final_dev (F32 [batch, H], optional)
 * receives the final norm's output.  Asynchronous on `stream`. */
NF_API int nf_stack_decode(nf_stack* stack, const int32_t* tokens_dev, const int32_t* positions_dev, int batch,
                           int32_t* next_dev, float* final_dev, void* stream);
/* Waits for `stream` and reports device-side failures (a token outside the
 * vocabulary, a position outside the cache, a bounded wait). */
NF_API int nf_stack_sync(nf_stack* stack, void* stream);

/* ---- router top-k without device allocation ------------------------------
 * No counterpart in the reference: its router runs inside moe() on host
 * buffers (src/text_forward.cpp:926-931).  This entry point is for callers
 * that cannot allocate device memory and so cannot create an nf_moe handle
 * (which owns weights and a workspace): a serving runtime whose memory pool
 * reserved the device's free memory up front, a path where a cudaMalloc
 * would synchronise the device, a process under a hard memory budget.
 *
 * Same routes as nf_moe_route (gemv_bf16 + router_select, bit-exact) from
 * caller-owned device buffers; nothing is allocated: the intermediate
 * logits, scores and choices live in a static device array compiled into
 * the library (about 192 KB of every device the library is used on).
 *   x_dev        BF16 [tokens, hidden], 16-byte aligned
 *   router_w_dev BF16 [experts, hidden], 16-byte aligned (mlp.gate.weight)
 *   bias_dev     F32  [experts] (mlp.gate.e_score_correction_bias)
 *   topk_idx_dev INT32 [tokens, top_k];  topk_w_dev F32 [tokens, top_k]
 *   msg, msg_len optional caller buffer that receives an error message
 * Limits: tokens x experts <= NF_NOALLOC_MAX_SCORES (e.g. 256 tokens at 64
 * experts); a larger call returns NF_ERR_CAPACITY before any device work.
 * hidden a multiple of 8, experts <= 1024, top_k <= 32.
 * The first call on a device does one-time set-up with that device current
 * (it resolves the scratch array's address and builds the sigmoid lookup
 * index, synchronising the device): make it before any stream capture.
 * Later calls only enqueue work on `stream`.  Every call on a device uses
 * the same scratch array, so calls that overlap in time (two streams, or two
 * threads, with no ordering between them) race and give wrong routes: order
 * them.  The chain always runs the separately rounded multiply and add (the
 * caller's weights are not range-checked), slower than nf_moe_route on large
 * batches.  If the logits stage gives up on its bounded wait, every
 * topk_idx entry of the call is -1. */
#define NF_NOALLOC_MAX_SCORES 16384
NF_API int nf_router_topk_noalloc(const uint16_t* x_dev, const uint16_t* router_w_dev, const float* bias_dev, int tokens,
                                  int hidden, int experts, int top_k, int n_group, int topk_group, int normalize,
                                  float routed_scaling, int32_t* topk_idx_dev, float* topk_w_dev, char* msg,
                                  int msg_len, void* stream);

#ifdef __cplusplus
}
#endif
#endif
