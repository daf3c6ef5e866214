/*
 * zonos2_cuda.h -- C ABI of the B200 (sm_100a) per-decode-step output path of
 * zonos2.cpp: the 9-codebook output head (hidden 2048 -> 9 x 1024 logits), the
 * tanh softcap 15*tanh(x/15) and the sampler (repetition penalty, temperature,
 * top-k / top-p / min-p, token masks, seeded categorical draw).
 *
 * Conventions
 *   - Every entry point returns int: >= 0 on success (a token id where the
 *     reference returned one), a negative ZONOS2CU_E* code on failure.  No C++
 *     exception crosses this boundary.
 *   - "_dev" pointers are CUDA device pointers owned by the caller; calls that
 *     take them are asynchronous and ordered on the cudaStream_t passed as
 *     `stream` (NULL = the legacy default stream).  "_host" pointers are host
 *     memory; those calls copy in and out and return when the result is on the
 *     host.
 *   - Device memory is allocated only by these calls:
 *       zonos2cu_ctx_create, zonos2cu_set_head, zonos2cu_set_allow,
 *       zonos2cu_set_out_norm, zonos2cu_set_embeddings, zonos2cu_gen_begin
 *         (owned by the context, freed by zonos2cu_ctx_destroy);
 *       the first zonos2cu_ctx_sample_host / zonos2cu_ctx_step_host of a
 *         context, and a later one with larger inputs (host-path staging,
 *         owned by the context);
 *       the first zonos2cu_sample_token on a device (a small per-device
 *         staging area, device and page-locked host memory, kept until exit);
 *       zonos2cu_comm_create and zonos2cu_comm_create_timeout (NCCL's own
 *         buffers, freed by zonos2cu_comm_destroy or zonos2cu_comm_abort);
 *       zonos2cu_ipc_alloc (freed by zonos2cu_ipc_free).
 *     Every other entry point, zonos2cu_step_noalloc included, allocates
 *     nothing.
 *   - Host buffers given to the "_host" calls are copied with
 *     cudaMemcpyAsync: page-locked memory (cudaHostAlloc, or
 *     cudaHostRegister on an existing buffer) copies at full PCIe speed,
 *     pageable memory (a plain std::vector) through a bounce buffer.
 *   - A context belongs to one device and is not thread-safe; use one per
 *     (device, host thread).
 *
 * Reference interfaces replaced (paths relative to the zonos2.cpp tree):
 *   sample_token(Xoshiro256&, const float*, int, float, int, float, float)
 *                                         src/zonos2_generate.cpp:36-93
 *   Xoshiro256 seeding / next / randf     src/zonos2_generate.cpp:11-33
 *   head: linear_forward(multi_output)    src/zonos2_model.cpp:200-216, :687-690
 *   softcap + [n_tok, 9, audio_vocab]     src/zonos2_model.cpp:692-703
 *   the per-step sampling loop            src/zonos2_generate.cpp:259-267
 */
#ifndef ZONOS2_CUDA_H
#define ZONOS2_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------- */
#define ZONOS2CU_OK 0
#define ZONOS2CU_EINVAL (-1)       /* an argument is out of range or NULL          */
#define ZONOS2CU_ECUDA (-2)        /* a CUDA runtime / driver call failed          */
#define ZONOS2CU_ENOMEM (-3)       /* a device allocation failed                   */
#define ZONOS2CU_ESTATE (-4)       /* context not ready (e.g. no head weights set) */
#define ZONOS2CU_EUNSUPPORTED (-5) /* shape outside what the kernels implement     */
#define ZONOS2CU_EDEVICE (-6)      /* a kernel reported a bounded wait that expired */
#define ZONOS2CU_ETOOBIG (-7)      /* larger than zonos2cu_step_noalloc's fixed scratch */
#define ZONOS2CU_ENCCL (-8)        /* NCCL is missing or an NCCL call failed        */

/* ---- per-row flags written next to each sampled code ---------------------- */
#define ZONOS2CU_FLAG_ALL_MASKED 1 /* no logit >= -1e9 survived: code = pad_id     */
#define ZONOS2CU_FLAG_NONFINITE 2  /* a NaN / +inf logit was treated as masked     */

typedef enum { ZONOS2CU_F32 = 0, ZONOS2CU_BF16 = 1 } zonos2cu_dtype;

/* Sampler knobs.  Meaning and defaults follow Zonos2GenParams
 * (src/zonos2.h:244-254).  repetition_penalty is build-defined (the reference
 * declares it but never reads it): every distinct token of the row's history
 * window is scaled once, l > 0 ? l * RN(1/rho) : l * rho; 1.0 disables it.
 * pad_id is the code forced by the delay-pattern mask and returned for
 * all-masked rows. */
typedef struct {
    float temperature; /* > 0                                    default 0.7  */
    int top_k;         /* <= 0 or >= vocab: off                  default 50   */
    float top_p;       /* >= 1: off                              default 0.9  */
    float min_p;       /* in [0, 1]; 0: off                      default 0.02 */
    float repetition_penalty; /* > 0; 1: off                     default 1.0  */
    int pad_id;        /* in [0, vocab)                          default 1023 */
} zonos2cu_sample_params;

/* Fills *p with the defaults above. */
void zonos2cu_default_params(zonos2cu_sample_params *p);

/* Library version string and the last CUDA error text seen on this thread. */
const char *zonos2cu_version(void);
const char *zonos2cu_last_error(void);

/* ---- generator ------------------------------------------------------------ */

/* Xoshiro256** seeded as the reference does (src/zonos2_generate.cpp:13-19):
 * state[i] = seed ^ K_i, then 20 discarded outputs.  Host-side helper. */
void zonos2cu_rng_seed(uint64_t seed, uint64_t state[4]);

/* ---- the drop-in for sample_token (src/zonos2_generate.cpp:36-37) --------- */

/* Same arguments and result as the reference's
 *   static int sample_token(Xoshiro256& rng, const float* logits,
 *                           int vocab_size, float temp, int top_k,
 *                           float top_p, float min_p);
 * rng_state are the generator's four state words (host memory), advanced by
 * exactly one draw; logits are vocab_size host floats (1 <= vocab_size <=
 * 1024).  The uniform is drawn on the host, as the reference draws it; the
 * row is sampled on the current CUDA device (one copy in, one launch, one copy
 * out).  Equal probabilities are taken in ascending token order.  Returns the
 * token id, or a negative ZONOS2CU_E* code (temp <= 0, NaN knobs, min_p > 1,
 * or an all-masked row -- the cases where the reference is undefined; the
 * generator is left unadvanced when the arguments are rejected). */
int zonos2cu_sample_token(uint64_t rng_state[4], const float *logits, int vocab_size,
                          float temp, int top_k, float top_p, float min_p);

/* ---- stateless batched sampler (device pointers) -------------------------- */

/* One decode step over n_streams x n_cb rows.  Row (s, c) is
 * logits_dev[(s*n_cb + c) * row_stride .. + vocab) (row_stride >= vocab; the
 * reference's [n_tok, 9, 1026] layout is row_stride = 1026).
 *   rng_dev      [n_streams][4] u64, 16-byte aligned: stream s draws one
 *                uniform per codebook,
 *                in codebook order (the reference's order at
 *                src/zonos2_generate.cpp:259-267), and is advanced by n_cb.
 *   hist_dev     [n_streams][n_cb][hist_len] i32 ring (may be NULL when
 *                hist_len == 0): read for the repetition penalty, then the
 *                sampled code is written at hist_pos.  Entries outside
 *                [0, vocab) are ignored (use -1 for empty slots).
 *   allow_dev    [n_streams][ceil(vocab/32)] u32 or NULL: bit t of stream s
 *                clear masks token t for all its codebooks.
 *   delay_step   >= 0: codebook c with delay_step < c may only emit pad_id
 *                (the delay pattern); < 0: off.
 *   codes_dev    [n_streams][n_cb] i32 output; flags_dev the same or NULL.
 * Limits: 1 <= vocab <= 1024, 1 <= n_cb <= 16. */
int zonos2cu_sample_rows(const float *logits_dev, int n_streams, int n_cb, int vocab,
                         long long row_stride, const zonos2cu_sample_params *params,
                         uint64_t *rng_dev, int32_t *hist_dev, int hist_len, int hist_pos,
                         const uint32_t *allow_dev, int delay_step, int32_t *codes_dev,
                         int32_t *flags_dev, void *stream);

/* ---- stateless output head + softcap (device pointers) -------------------- */

/* logits_dev[b][c][v] = softcap * tanh(dot(hidden[b], W[c*rows_per_cb + v]) / softcap)
 * for b < batch, c < n_cb, v < vocab (softcap <= 0: no cap).  W_dev is the
 * head weight [n_cb*rows_per_cb][dim] row-major -- the reference's
 * multi_output / output.bin layout is rows_per_cb = 1026, vocab = 1024
 * (src/zonos2_loader.cpp:133-136) -- and hidden_dev is [batch][dim], both of
 * `dtype`.  F32 runs an f32-exact GEMV (f64 accumulation); BF16 runs the
 * tcgen05 tensor-core GEMM (f32 accumulation in TMEM) and needs
 * dim % 64 == 0, vocab % 64 == 0 and 16-byte aligned rows. */
int zonos2cu_head_softcap(const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb, int n_cb,
                          int vocab, int dim, const void *hidden_dev, int batch, float softcap,
                          float *logits_dev, void *stream);

/* ---- context: device-resident state for a batch of decode streams --------- */

typedef struct zonos2cu_ctx zonos2cu_ctx;

typedef struct {
    int n_streams;   /* decode streams held by this context (this device's shard) */
    int n_cb;        /* codebooks per frame: 9                                     */
    int vocab;       /* sampled tokens per codebook: 1024                          */
    int dim;         /* hidden size for the fused head: 2048 (0: sampler only)     */
    int hist_len;    /* repetition-history window per row (0: none; <= 65535)      */
    uint64_t seed;   /* stream s uses Xoshiro256(seed + first_stream + s)          */
    uint64_t first_stream; /* global index of this shard's first stream           */
} zonos2cu_dims;

int zonos2cu_ctx_create(int device, const zonos2cu_dims *dims, zonos2cu_ctx **out);
int zonos2cu_ctx_destroy(zonos2cu_ctx *ctx);

/* The setters and getters below synchronise the device: they are set-up calls,
 * safe against steps enqueued on any stream, not per-step calls. */

/* Head weights from host memory, [n_cb*rows_per_cb][dim] of dtype
 * (rows_per_cb = 1026 for the reference's output.bin; only the first vocab
 * rows of each codebook are kept on the device). */
int zonos2cu_set_head(zonos2cu_ctx *ctx, const void *W_host, zonos2cu_dtype dtype,
                      int rows_per_cb);
/* History ring [n_streams][n_cb][hist_len] and its write position.  The
 * context also keeps, per row, how often each token occurs in the ring and a
 * bitmap of the tokens present, updated by every step for the token it evicts
 * and the one it appends: the penalty reads 128 bytes per row instead of the
 * whole ring. */
int zonos2cu_set_history(zonos2cu_ctx *ctx, const int32_t *hist_host, int hist_pos);
int zonos2cu_get_history(zonos2cu_ctx *ctx, int32_t *hist_host, int *hist_pos);
/* Generator states [n_streams][4]. */
int zonos2cu_set_rng(zonos2cu_ctx *ctx, const uint64_t *state_host);
int zonos2cu_get_rng(zonos2cu_ctx *ctx, uint64_t *state_host);
/* Allow bitmask [n_streams][ceil(vocab/32)]; NULL clears it. */
int zonos2cu_set_allow(zonos2cu_ctx *ctx, const uint32_t *bits_host);

/* The output RMSNorm ahead of the head in zonos2cu_ctx_step: replaces
 * rms_norm_per_token(x, dim, n, eps, out_norm.weight) applied to the last hidden
 * states before the multi_output head (src/zonos2_model.cpp:684-685, :19-35).
 * With it enabled, ctx_step takes the un-normalised hidden states.  weight_host
 * is [dim] f32, or NULL for no scale weight; enable = 0 turns it off.  With an
 * f32 head the norm is the reference's, exactly; with a bf16 head it is folded
 * into the head (the weight into W's columns, rounded to bf16 once; each row's
 * 1 / rms into the GEMM's epilogue), within the bf16 path's tolerance. */
int zonos2cu_set_out_norm(zonos2cu_ctx *ctx, int enable, const float *weight_host, float eps);
/* Classifier-free guidance in zonos2cu_ctx_step: the blend
 * uncond + scale * (cond - uncond) of softcapped logits that the reference
 * applies to its prefill logits (src/zonos2_generate.cpp:157-183), here on every
 * step.  With it enabled, ctx_step and ctx_step_host take [2*n_streams][dim]
 * hidden states, row 2s the conditional and row 2s+1 the unconditional state
 * of stream s; logits and codes stay [n_streams][...].  enable = 0 turns it off. */
int zonos2cu_set_cfg(zonos2cu_ctx *ctx, int enable, float scale);

/* One sampling step from device logits [n_streams][n_cb][row_stride] on
 * `stream` (NULL = the legacy default stream, like every "_dev" call); the
 * history position advances by one (mod hist_len) on success.  The host-path
 * calls below run on the context's own stream (zonos2cu_ctx_stream): work a
 * caller enqueues on other streams is not ordered with them, so synchronise
 * between the two kinds of call.  Each step reads what the step before it wrote
 * (generator states, history, the uniforms drawn ahead): a context's steps go on
 * one stream, or on streams the caller orders with events. */
int zonos2cu_ctx_sample(zonos2cu_ctx *ctx, const float *logits_dev, long long row_stride,
                        const zonos2cu_sample_params *params, int delay_step,
                        int32_t *codes_dev, int32_t *flags_dev, void *stream);
/* The same from host logits [n_streams][n_cb][row_stride] to host codes/flags
 * (flags may be NULL): copies in, samples, copies out, returns when done. */
int zonos2cu_ctx_sample_host(zonos2cu_ctx *ctx, const float *logits_host, long long row_stride,
                             const zonos2cu_sample_params *params, int delay_step,
                             int32_t *codes_host, int32_t *flags_host);
/* One fused step: hidden [n_streams][dim] (device, dtype; [2*n_streams][dim] with
 * guidance on) -> output RMSNorm if set -> head + softcap -> guidance blend if
 * set -> sampler.  logits_out_dev ([n_streams][n_cb][vocab] f32) may be NULL. */
int zonos2cu_ctx_step(zonos2cu_ctx *ctx, const void *hidden_dev, zonos2cu_dtype dtype,
                      const zonos2cu_sample_params *params, int delay_step, int32_t *codes_dev,
                      int32_t *flags_dev, float *logits_out_dev, void *stream);
/* The same from host hidden states to host codes. */
int zonos2cu_ctx_step_host(zonos2cu_ctx *ctx, const void *hidden_host, zonos2cu_dtype dtype,
                           const zonos2cu_sample_params *params, int delay_step,
                           int32_t *codes_host, int32_t *flags_host);
/* The context's CUDA stream (cudaStream_t), for callers that order work on it. */
void *zonos2cu_ctx_stream(zonos2cu_ctx *ctx);

/* ---- the generation loop around the step ------------------------------------
 * Replaces the frame bookkeeping of zonos2_generate's loop
 * (src/zonos2_generate.cpp:203-279) for a batch: between zonos2cu_gen_begin and
 * zonos2cu_gen_end, every zonos2cu_ctx_sample / zonos2cu_ctx_step (and their
 * host variants) also keeps the step's frame on the device, on the step's
 * stream: codes clamped to vocab - 1 (:214, :264), the stream ended after the
 * first frame holding eoa_id (:218-224, :269-276; that frame is kept), at most
 * max_frames frames per stream, and the next step's input frame (the codes,
 * then text_pad_id; :238-243).  With the reference's constants (1024 sampled
 * tokens, eoa_id 1024) no frame can hold eoa_id, so streams run to max_frames,
 * as in the reference.  gen_begin clears the state; before the first frame the
 * next input frame is audio_pad_id codes and text_pad_id. */
int zonos2cu_gen_begin(zonos2cu_ctx *ctx, int max_frames, int eoa_id, int audio_pad_id,
                       int text_pad_id);
int zonos2cu_gen_end(zonos2cu_ctx *ctx);
/* Frames [n_streams][max_frames][n_cb] (entries past a stream's count are -1),
 * frame counts [n_streams], end-of-audio frame [n_streams] (-1: none); any
 * pointer may be NULL.  Synchronises the device. */
int zonos2cu_gen_read(zonos2cu_ctx *ctx, int32_t *frames_host, int32_t *n_frames_host,
                      int32_t *eos_at_host);
/* Device pointer to the next step's input frames [n_streams][n_cb + 1] (NULL
 * before gen_begin). */
const int32_t *zonos2cu_gen_next_input(zonos2cu_ctx *ctx);
/* shear_up of every stream's frames (scripts/dac_decode.py:23-30): out_dev
 * [n_streams][max_frames][n_cb], out[s][t][j] = frames[s][t + j][j] while
 * t + j < the stream's frame count, audio_pad_id elsewhere. */
int zonos2cu_gen_shear_up(zonos2cu_ctx *ctx, int32_t *out_dev, void *stream);
/* The model's input embedding tables, f32 row-major: codebook tables
 * [n_cb][audio_vocab][dim] (Zonos2Weights::codebook_embeds) and the text table
 * [text_vocab + 1][dim] (text_embed, padding row last). */
int zonos2cu_set_embeddings(zonos2cu_ctx *ctx, const float *codebook_tables_host,
                            const float *text_table_host, int audio_vocab, int text_vocab);
/* embedding_sum (src/zonos2_model.cpp:116-151) of the next input frames into
 * out_dev [n_streams][dim] f32: the next model step's input. */
int zonos2cu_gen_embed_next(zonos2cu_ctx *ctx, float *out_dev, void *stream);
/* The same on caller buffers: ids_dev [n_frames][n_cb + 1], out_dev [n_frames][dim]. */
int zonos2cu_embed_frames(const float *codebook_tables_dev, const float *text_table_dev,
                          int n_cb, int audio_vocab, int text_vocab, int dim,
                          const int32_t *ids_dev, int n_frames, float *out_dev, void *stream);
/* Writes frames_host [n_frames][n_cb] in the reference's codes.bin format
 * (decode_dac_to_wav, src/zonos2_generate.cpp:285-306): int32 n_frames, int32
 * n_cb, then the codes frame by frame. */
int zonos2cu_write_codes_bin(const char *path, const int32_t *frames_host, int n_frames,
                             int n_cb);

/* Reads and clears the device-side error word that bounded waits set when
 * they expire (synchronises the current device).  0 = no error. */
int zonos2cu_device_error(void);

/* ---- several GPUs: batch-sharded streams, codes collected on one rank --------
 * One process per GPU.  Rank r of n owns the contiguous slice [first, first +
 * count) of the global batch that zonos2cu_shard_range gives (the first
 * n_streams % n_ranks ranks own one stream more) and creates its context with
 * that count and first_stream = first: its generators and codes then equal the
 * same streams of a one-GPU run of the whole batch.  Nothing crosses GPUs but
 * the codes, which the writer rank collects -- the frame collection of
 * src/zonos2_generate.cpp:278, for a batch.  NCCL is loaded at run time
 * (libnccl.so.2, or the copy the process already holds); without it these
 * calls return ZONOS2CU_ENCCL and the rest of the library is unaffected. */
int zonos2cu_shard_range(long long n_streams, int n_ranks, int rank, long long *first,
                         long long *count);
/* An NCCL communicator over the job's ranks (a ncclComm_t, as void *): rank 0
 * makes the id, the caller hands it to every rank out of band (MPI, a file, a
 * socket), then every rank calls zonos2cu_comm_create with it -- collectively,
 * as ncclCommInitRank is.  A caller that has its own NCCL communicator passes
 * that to zonos2cu_gather_codes instead. */
int zonos2cu_comm_unique_id(unsigned char id[128]);
int zonos2cu_comm_create(int device, int n_ranks, int rank, const unsigned char id[128],
                         void **nccl_comm_out);
/* The same communicator, set up without blocking (ncclCommInitRankConfig with
 * blocking = 0) and polled: if every rank has not joined within timeout_ms the
 * set-up is aborted (ncclCommAbort) and ZONOS2CU_ENCCL returned, so a rank that
 * died or never started cannot hang the others in set-up.  Its gathers wait at
 * most 120 s for connections and its destroy at most 60 s for the flush (then
 * aborts).  Needs NCCL >= 2.14; otherwise ZONOS2CU_ENCCL. */
int zonos2cu_comm_create_timeout(int device, int n_ranks, int rank, const unsigned char id[128],
                                 int timeout_ms, void **nccl_comm_out);
/* Flushes (a communicator from zonos2cu_comm_create_timeout, within 60 s) and
 * frees a communicator. */
int zonos2cu_comm_destroy(void *nccl_comm);
/* Frees a communicator at once, ending the operations still in flight on it
 * (ncclCommAbort): the error path when a peer rank is known to be gone. */
int zonos2cu_comm_abort(void *nccl_comm);
/* Collects n_steps steps of codes on rank `root`, called by every rank of the
 * communicator with the same root, n_steps, n_streams (the global batch) and
 * n_cb, on `stream` (asynchronous; nothing is synchronised).  codes_dev is this
 * rank's block [n_steps][count][n_cb] (e.g. a ring of per-step codes); out_dev
 * (root only; others may pass NULL) receives every rank's block in rank
 * order: rank r's at element n_steps * first_r * n_cb.  For n_steps = 1 that
 * is the global [n_streams][n_cb].  Only the root receives: the other ranks
 * send and return. */
int zonos2cu_gather_codes(void *nccl_comm, int root, const int32_t *codes_dev, int n_steps,
                          long long n_streams, int n_cb, int32_t *out_dev, void *stream);

/* The same collection by the copy engines, for a loop that must not give SMs or
 * a collective to it: the root allocates its output with zonos2cu_ipc_alloc
 * (device memory of the library's own, freed by zonos2cu_ipc_free) and hands
 * the 64-byte handle to every other rank out of band; each of those maps it
 * once with zonos2cu_ipc_open (a pointer into the root's GPU, valid in this
 * process until zonos2cu_ipc_close) and, after each block of steps, enqueues
 * zonos2cu_push_codes of its codes to their place in the root's output, on a
 * stream ordered after those steps.  The copies run on the copy engines over
 * NVLink while the SMs run the next steps; no rank waits for another in the
 * loop.  The caller orders the reuse of its source buffer after the copy (an
 * event) and, before the root reads its output, the completion of every rank's
 * copies (each rank synchronises its copy stream, then a barrier).  All on one
 * node. */
int zonos2cu_ipc_alloc(int device, long long bytes, void **dev_ptr_out, unsigned char handle[64]);
int zonos2cu_ipc_free(void *dev_ptr);
int zonos2cu_ipc_open(int device, const unsigned char handle[64], void **dev_ptr_out);
int zonos2cu_ipc_close(void *dev_ptr);
/* n_steps blocks of elems_per_step int32 codes, contiguous in codes_dev (e.g.
 * [n_steps][count][n_cb] of a ring), to dst_dev + k * dst_stride for block k
 * (e.g. rank r's place, first_r * n_cb, in the root's [n_steps][n_streams][n_cb]
 * output: dst_stride = n_streams * n_cb), one strided copy asynchronous on
 * `stream`.  Pushing a block of steps at a time keeps the step stream free of
 * per-step event waits, which would cut the programmatic overlap of one step's
 * launch with the step before. */
int zonos2cu_push_codes(const int32_t *codes_dev, int n_steps, long long elems_per_step,
                        int32_t *dst_dev, long long dst_stride, void *stream);

/* ---- one decode step that allocates nothing -------------------------------- */

/* No counterpart in the reference.  For callers that may not allocate device
 * memory -- a host application whose device memory belongs to another
 * framework's pool, or a real-time decode loop where an allocation could
 * block or synchronise the device.  It runs zonos2cu_head_softcap and then
 * zonos2cu_sample_rows (same arguments, same results) with the intermediate
 * logits in a fixed device array compiled into the library: every GPU that
 * loads the library holds ZONOS2CU_NOALLOC_MAX_LOGITS floats (2.25 MiB) of it
 * until the process exits, and no call allocates or frees anything.
 *   - n_streams * n_cb * vocab must not exceed ZONOS2CU_NOALLOC_MAX_LOGITS
 *     (64 streams of 9 x 1024): larger requests return ZONOS2CU_ETOOBIG.
 *   - The array's device address belongs to the CUDA context current at the
 *     call.  Outside stream capture each call looks it up (cudaGetSymbolAddress,
 *     which allocates nothing); a call made while `stream` is capturing uses
 *     the address found by the last call outside capture in the same context,
 *     and returns ZONOS2CU_ESTATE if that context has made none.  So make one
 *     call in a context before capturing it, and again after cudaDeviceReset.
 *   - All calls on a device share the one array: calls whose work overlaps on
 *     the GPU race.  Order them on one stream, or synchronise between them.
 *   - Every argument is checked before anything is launched, as the two entry
 *     points would check it (n_streams = 0 included).
 * Arguments are those of the two entry points it combines (softcap 15 in
 * the model; row stride of the logits = vocab). */
#define ZONOS2CU_NOALLOC_MAX_LOGITS (64 * 9 * 1024)
int zonos2cu_step_noalloc(const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb, int n_cb,
                          int vocab, int dim, const void *hidden_dev, int n_streams, float softcap,
                          const zonos2cu_sample_params *params, uint64_t *rng_dev,
                          int32_t *hist_dev, int hist_len, int hist_pos,
                          const uint32_t *allow_dev, int delay_step, int32_t *codes_dev,
                          int32_t *flags_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* ZONOS2_CUDA_H */
