/* g4: B200-native (sm_100a) speculative greedy-decode hot path behind a thin C ABI.
 *
 * Drop-in boundary for the kernel-header operator surface of gemma4-e2b-laptop-cpu
 * (engine/w4g32_avx2.h, engine/w4a8_avx2.h, engine/bf16_exp3_head.h and the engine tasks in
 * engine/gemma4_engine.cpp).  Every entry point takes plain pointers and sizes, returns an int
 * status (G4_OK or a negative G4_ERR_*; g4_last_error() gives the message), never allocates,
 * and enqueues its work on the CUDA stream passed as `stream` (NULL = the legacy default
 * stream).  Pointers marked "dev" are device memory; all others are host memory.
 *
 * Layouts (identical to the reference unless stated):
 *   W4 weights   uint8  [N][K/2]   two int4 values (q+8) per byte; the reference layout has low
 *                                  nibble = even k (w4g32_avx2.h:1-6); the device layout made by
 *                                  g4_w4_pack has, per 32-group, byte b = element b (low nibble)
 *                                  and element 16+b (high nibble).
 *   W4 scales    bf16   [N][K/32]
 *   activations  fp32   [M][K]     row m at X + m*K; outputs Y[m*ldy + n]
 *   int8 acts    int8   [M][K], scales fp32 [M][K/32], sums int32 [M][K/32]  (w4a8_avx2.h:29)
 *   bf16-exp3    44 B per 32-group (bf16_exp3_head.h:1-4) + CSR exceptions (exc_ptr int64[N+1],
 *                exc_col uint16, exc_delta fp32)
 *   KV cache     bf16   [ctx][hd]  one KV head (gemma4_engine.cpp:1248)
 * K must be a multiple of 32 everywhere (256 for the GEMMs).
 */
#ifndef G4_H
#define G4_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4_OK 0
#define G4_ERR_INVALID (-1)     /* bad argument (size, alignment, null pointer) */
#define G4_ERR_CUDA (-2)        /* a CUDA call failed */
#define G4_ERR_TIMEOUT (-3)     /* a device-side wait gave up (status word set by the kernel) */
#define G4_ERR_NOMEM (-4)       /* caller-provided workspace too small */
#define G4_ERR_UNSUPPORTED (-5) /* shape outside what this build supports */

/* Message of the last failed call on this host thread. */
const char* g4_last_error(void);
/* ABI version of this library (bumped on any signature change). */
int g4_abi_version(void);
/* Device status word (OR over the library's kernels on the current device): bit 0 set when a
 * device-side bounded wait gave up; bit 1 set when a CTA then returned while its own bulk copies
 * or tensor-core operations could still be in flight (a second bounded wait for them gave up too),
 * so memory a later CTA owns may have been written.  Once a call has returned bit 1, every
 * launching entry point fails with G4_ERR_TIMEOUT until a call with reset != 0.  Synchronous;
 * reset != 0 clears the word. */
int g4_device_status(unsigned* out, int reset);

/* ---------------------------------------------------------------- W4G32 / W4A8 linears */

/* Load-time relayout of reference W4 weights (the role of w4a8::repack_tiles,
 * w4a8_avx2.h:20-27): W dev [N][K/2] reference layout -> Wp dev [N][K/2] device layout. */
int g4_w4_pack(const uint8_t* W, int N, int K, uint8_t* Wp, void* stream);

/* Per-32-group sequential sums of X (the gsum half of w4::prep_x, w4g32_avx2.h:20-23):
 * X dev [M][K] -> gsum dev [M][K/32]. */
int g4_w4g32_gsum(const float* X, int M, int K, float* gsum, void* stream);

/* Float-activation int4 GEMM, Y[m*ldy+n] = sum_g s[n,g]*(sum_i t*x - 8*gsum) in the exact fp32
 * order of w4::gemm_rows_tile<MT> (w4g32_avx2.h:65-96) as dispatched by lin_task/lin_multi
 * (gemma4_engine.cpp:243-255, 310-317).  Wp dev (device layout), S dev, X dev, gsum dev or NULL
 * (then computed in-kernel), Y dev.  1 <= M <= 8, K % 256 == 0. */
int g4_w4g32_gemm(const uint8_t* Wp, const uint16_t* S, const float* X, const float* gsum, int M, int N,
                  int K, float* Y, int ldy, void* stream);

/* Per-(row, 32-group) symmetric int8 quantisation, bit-exact to w4a8::quant (w4a8_avx2.h:30-42).
 * X dev [M][K] -> q dev [M][K], sx dev [M][K/32], sum dev [M][K/32]. */
int g4_w4a8_quant(const float* X, int M, int K, int8_t* q, float* sx, int32_t* sum, void* stream);

/* Int8-activation int4 GEMM, integer-exact group dots and the fp32 scale chain of
 * w4a8::tile<MT> (w4a8_avx2.h:46-60) / i8_task (gemma4_engine.cpp:304-309).
 * Wp dev (device layout), S dev, q/sx/sum dev (from g4_w4a8_quant), Y dev.  1 <= M <= 8. */
int g4_w4a8_gemm(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, const int32_t* sum,
                 int M, int N, int K, float* Y, int ldy, void* stream);

/* Workspace bytes of g4_w4a8_gemm_tc. */
size_t g4_w4a8_gemm_tc_ws_bytes(int M, int N, int K);
/* g4_w4a8_gemm for any M on the tensor cores (tcgen05.mma kind::i8, the prefill path of the
 * reference's fwd blocks, gemma4_engine.cpp:1595-1599 -> w4a8::tile<MT>, w4a8_avx2.h:46-60): the
 * same integer group dots (s8 weights q = t - 8 against the int8 activations) and the same fp32
 * chain per (row, activation row), so the same bits.  Wp dev (device layout), S dev, q dev [M][K],
 * sx dev [M][K/32] (the group sums are not needed), Y dev [M][ldy]; ws dev of
 * g4_w4a8_gemm_tc_ws_bytes() (256-byte aligned: the s8 weights and transposed scales are built in
 * it on every call).  N and K multiples of 128. */
int g4_w4a8_gemm_tc(const uint8_t* Wp, const uint16_t* S, const int8_t* q, const float* sx, int M, int N, int K, float* Y,
                    int ldy, void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------- row norms */

/* RMS norm of M rows, y = (x * r) * w with r = 1 / sqrtf((float)(ss / n) + 1e-6f) and ss the sum
 * of squares in double over the reference's 16 ordered partials (rms / rms_prep_x,
 * gemma4_engine.cpp:326-352, 365-381); y rounded to bf16 when round != 0.  When q is not NULL the
 * rows of y are also quantised as g4_w4a8_quant does (q [M][n], sx and sum [M][n/32]).
 * x, w, y dev; n a multiple of 256, at most 2048. */
int g4_rmsnorm(const float* x, const float* w, int M, int n, float* y, int round, int8_t* q, float* sx, int32_t* sum,
               void* stream);

/* ---------------------------------------------------------------- output head */

/* Once per device, before any stream capture: uploads the softcap table (r16(30*tanh(s/30)) of
 * every bf16 value, computed with the host libm) that the head entry points use. */
int g4_device_init(void);

/* Codebook of the bf16-exp3 head: the 8 most frequent exponents of E (stable order by count),
 * gemma4_engine.cpp:1232-1234.  E dev bf16 [count]; cb8 host [8]; ws dev >= 2048 B.  Synchronous. */
int g4_bf16p_codebook(const uint16_t* E, long long count, uint8_t* cb8, void* ws, size_t ws_bytes, void* stream);
/* First half of bf16p::pack (bf16_exp3_head.h:26-49): exceptions per row, exclusive-scanned into
 * exc_ptr dev [N+1]; *total (host) = exception count.  ws dev >= 8*N B.  Synchronous. */
int g4_bf16p_count(const uint16_t* E, int N, int K, const uint8_t* cb8, long long* exc_ptr, void* ws, size_t ws_bytes,
                   long long* total, void* stream);
/* Second half: the 44-byte groups (data dev [N*K/32*44]) and the CSR exceptions (exc_col dev,
 * exc_delta dev, sized by g4_bf16p_count), byte-identical to bf16p::pack. */
int g4_bf16p_pack(const uint16_t* E, int N, int K, const uint8_t* cb8, uint8_t* data, const long long* exc_ptr,
                  uint16_t* exc_col, float* exc_delta, void* stream);
/* Raw head logits Y[m*ldy+n] (before bf16 rounding) in the fp32 order of bf16p::rows_tile
 * (bf16_exp3_head.h:84-107) / head_task (gemma4_engine.cpp:574-579).  X dev [M][K], M <= 4. */
int g4_bf16p_gemm(const uint8_t* data, const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col,
                  const float* exc_delta, int N, int K, const float* X, int M, float* Y, int ldy, void* stream);
/* B200 copy of a packed head in the unpacked layout: per group the 32 weights as bf16p::pack
 * represents them (codebook exponent, before the exception patches) as bf16, 64 bytes per group,
 * bytes 32h..32h+31 holding the weights of half h (octets in the order 0, 2, 1, 3, elements
 * 8o+4h..8o+4h+3 of octet o).  data dev (g4_bf16p_pack), cb8 host -> unp dev [N*K/32*64], 16-byte
 * aligned. */
int g4_bf16p_unpack(const uint8_t* data, const uint8_t* cb8, int N, int K, uint8_t* unp, void* stream);
/* g4_bf16p_gemm over the unpacked copy and the same exceptions: the same values (K a multiple of 64). */
/* Split-nibble copy of a packed head (48 B per group: the sign/mantissa bytes [N][G/4][2][4][16] —
 * per 4 groups the half-0 parts, then the half-1 parts — then the 3-bit exponent codes as nibbles
 * [N][G][16]), in the order the full-head GEMV consumes them (K % 128 == 0):
 * 25% fewer bytes than the unpacked copy, decoded with byte permutes over the codebook.  nib dev
 * [g4_bf16p_nib_bytes(N, K)], 16-byte aligned. */
size_t g4_bf16p_nib_bytes(int N, int K);
int g4_bf16p_nib_pack(const uint8_t* data, int N, int K, uint8_t* nib, void* stream);
/* The exact-head GEMV over the split-nibble copy (K % 128 == 0, M <= 4): the values of
 * g4_bf16p_gemm. */
int g4_bf16p_nib_gemm(const uint8_t* nib, const uint8_t* cb8, const long long* exc_ptr, const uint16_t* exc_col,
                      const float* exc_delta, int N, int K, const float* X, int M, float* Y, int ldy, void* stream);
int g4_bf16p_unpacked_gemm(const uint8_t* unp, const long long* exc_ptr, const uint16_t* exc_col, const float* exc_delta,
                           int N, int K, const float* X, int M, float* Y, int ldy, void* stream);
/* Greedy pick over raw logits: r16, max, then the lowest index whose softcapped value equals the
 * max's (gemma4_engine.cpp:1491-1497).  out_idx dev [M]; ws dev >= 8*M B. */
int g4_head_argmax(const float* Y, int M, int N, int ldy, int* out_idx, void* ws, size_t ws_bytes, void* stream);
/* Int4 screen copy of the head: device W4 layout (see g4_w4_pack), bf16 scales f2bf(amax/7) and
 * the per-row error coefficient (gemma4_engine.cpp:1235-1244, for any K). */
int g4_screen_build(const uint16_t* E, int N, int K, uint8_t* W4p, uint16_t* S4, float* coef, void* stream);
size_t g4_head_screen_ws_bytes(int M, int N, int lim);
/* Certified screen + exact rescoring + pick for M <= 4 hidden rows H dev [M][K]
 * (screen_task :460-538, eval_row :1453-1474, resc_task :540-571), all on the device; more than
 * lim survivors (the reference uses 30000) falls back to the full exact head, as the reference
 * does.  out_idx dev [M] winners; out_nsurv dev [M] survivor counts (-1 = fallback). */
int g4_head_screen(const uint8_t* W4p, const uint16_t* S4, const float* coef, const uint8_t* data, const uint8_t* cb8,
                   const long long* exc_ptr, const uint16_t* exc_col, const float* exc_delta, int N, int K,
                   const float* H, int M, int lim, int* out_idx, int* out_nsurv, void* ws, size_t ws_bytes,
                   void* stream);

/* Vocab-parallel screen (one shard of N head rows per device, rows row0.. of the full head): the
 * single-device screen split at its two global reductions.  Per call, with M <= 4 rows of H:
 *   1. g4_head_screen_shard_bound: screen GEMV and the shard's bound L_out dev [M];
 *   2. the caller reduces L across the shards (max) into L;
 *   3. g4_head_screen_shard_select: survivors against the global threshold, exact rescoring or (on
 *      overflow) the shard's full exact head (unp may be NULL: the bf16p rows are read), and the
 *      shard's largest candidate value vmax_out dev [M]; out_nsurv dev [M] (-1 = fallback);
 *   4. the caller reduces vmax across the shards (max) into gmax;
 *   5. g4_head_screen_shard_pick: the shard's lowest global index whose candidate value v has
 *      v >= gmax - 2 and the same softcapped value as gmax, or INT_MAX; idx_out dev [M];
 *   6. the caller reduces the indices (min); INT_MAX means no winner (-1).
 * ws as for g4_head_screen (g4_head_screen_ws_bytes(M, N, lim)), kept between the phases. */
int g4_head_screen_shard_bound(const uint8_t* W4p, const uint16_t* S4, const float* coef, int N, int K, const float* H,
                               int M, int lim, float* L_out, void* ws, size_t ws_bytes, void* stream);
int g4_head_screen_shard_select(const float* coef, const uint8_t* data, const uint8_t* unp, const uint8_t* cb8,
                                const long long* exc_ptr, const uint16_t* exc_col, const float* exc_delta, int N, int K,
                                const float* H, int M, int lim, const float* L, float* vmax_out, int* out_nsurv, void* ws,
                                size_t ws_bytes, void* stream);
int g4_head_screen_shard_pick(int N, int M, int lim, int row0, const float* gmax, int* idx_out, void* ws, size_t ws_bytes,
                              void* stream);

/* The vocab-parallel screen in one call over an NCCL communicator (one process per GPU, rank r
 * holding rows row0.. of the head), on `stream`: broadcast of H (dev [M][K]) from root, the
 * shard's bound, all-reduce max, survivors / rescoring or the shard's exact head, all-reduce max of
 * the candidate value, the shard's pick, all-reduce min -> out_idx dev [M] (the same winners on every
 * rank, -1 = none).  Shard arguments as for g4_head_screen_shard_*; ws dev of
 * g4_head_screen_dist_ws_bytes (256-byte aligned).  Every step is a stream operation: the call can
 * be recorded in a CUDA graph.  The reference screens on one host (screen_task :460-538, eval_row
 * :1453-1474); this is its vocab-parallel form. */
size_t g4_head_screen_dist_ws_bytes(int M, int N, int lim);
int g4_head_screen_dist(void* nccl_comm, int root, const uint8_t* W4p, const uint16_t* S4, const float* coef,
                        const uint8_t* data, const uint8_t* unp, const uint8_t* cb8, const long long* exc_ptr,
                        const uint16_t* exc_col, const float* exc_delta, int N, int K, int row0, float* H, int M, int lim,
                        int* out_idx, void* ws, size_t ws_bytes, void* stream);
/* NCCL communicators for g4_head_screen_dist (NCCL is loaded on first use: libnccl.so.2, the copy
 * already in the process when there is one): a 128-byte unique id made on one rank and shared by
 * the caller, a communicator per rank on the current device, and its destruction. */
int g4_nccl_get_unique_id(void* id128);
int g4_nccl_comm_init(const void* id128, int nranks, int rank, void** comm);
int g4_nccl_comm_destroy(void* comm);

/* ---------------------------------------------------------------- split-KV decode attention */

/* Workspace bytes g4_attn_splitkv needs for these sizes. */
size_t g4_attn_splitkv_ws_bytes(int M, int nh, int hd, int kmin, int kmax, int T);

/* Decode/verify attention of M <= 4 query rows, nh <= 8 query heads over one bf16 KV head, keys
 * kmin..kmax split into T chunks as the reference's pool threads split them (attn_task,
 * gemma4_engine.cpp:743-877) and merged with its exact log-sum-exp rescale (attn_merge
 * :1019-1059).  Row m attends keys lo[m]..pos[m] (host arrays).  Kc, Vc dev bf16 [ctx][hd];
 * q dev fp32 [M][nh][hd] (softmax scale already folded in); out dev fp32 [M][nh][hd], values
 * rounded to bf16; ws dev scratch of g4_attn_splitkv_ws_bytes(); hd % 32 == 0, hd <= 512. */
int g4_attn_splitkv(const uint16_t* Kc, const uint16_t* Vc, const float* q, const int* pos, const int* lo, int M,
                    int nh, int hd, int kmin, int kmax, int T, float* out, void* ws, size_t ws_bytes, void* stream);

/* Same computation as g4_attn_splitkv for callers that cannot allocate device memory or hand over
 * a workspace (an embedding host whose arena owns all device memory, or a latency-critical decode
 * thread that must not risk the device-wide synchronisation a cudaMalloc/cudaFree can cause).
 * No counterpart in the reference.  Scratch is a fixed device global inside libg4.so (1,312,768
 * bytes, held by every GPU that loads the library until exit); limits: hd <= 256, T <= 8,
 * kmax - kmin + 1 <= 8192 keys (plus M <= 4, nh <= 8), larger calls return G4_ERR_UNSUPPORTED.
 * The first call on a device looks up the scratch address (cudaGetSymbolAddress) with that device
 * current: make it before any stream capture.  Calls share the scratch, so calls that overlap on
 * the GPU race; serialise them. */
int g4_attn_splitkv_noalloc(const uint16_t* Kc, const uint16_t* Vc, const float* q, const int* pos, const int* lo,
                            int M, int nh, int hd, int kmin, int kmax, int T, float* out, void* stream);

/* ---------------------------------------------------------------- speculative decode engine */

/* The synthetic Gemma-style E2B model of BASELINE.json configs[4] (dimensions and seeded weights
 * in gemma4-e2b-laptop-cpu_b200/csrc/g4_model.cuh) with its MTP drafter, prompt lookup, batched
 * verification and greedy acceptance: the reference's run_req / fwd / draft_step
 * (gemma4_engine.cpp:1582-1663, 1256-1502, 1534-1563) in chain mode. */
typedef struct g4_engine g4_engine;
typedef struct {
  int hidden, n_layers, mlp, vocab;  /* 2048, 30, 8192, 262144 (vocab a power of two, = 128 x centroids) */
  int ctx_max;                       /* KV cache positions */
  int prefill_block;                 /* ENGINE_PREFILL_BLOCK (32) */
  int k_draft;                       /* ENGINE_K (3) */
  int ngram, ngram_len;              /* ENGINE_NGRAM (2), ENGINE_NGLEN (3) */
  int prefill_int8, decode_int8;     /* ENGINE_PREFILL_INT8 (1), ENGINE_DECODE_INT8 (1) */
  int head_screen, screen_lim;       /* ENGINE_HEAD_SCREEN: 0 = the full exact head every pass, 1 = the
                                        certified screen every pass (the reference), 2 = the screen
                                        with back-off (the default): after a pass whose screen fell
                                        back, the next 1, 2, 4 .. 64 passes go straight to the full
                                        exact head; same tokens in all three.  Survivor limit (30000) */
  int attn_chunks;                   /* split-KV key chunks = the reference's pool threads (8) */
  int att_par;                       /* ENGINE_ATT_PAR (192) */
  int drafter;                       /* build the MTP drafter (1) */
  unsigned long long seed;           /* weight seed */
  int graphs;                        /* decode rounds as CUDA graphs with programmatic dependent
                                        launch (1), graphs with ordinary launches (2), eager (0) */
  int fused_layers;                  /* verify passes on the int8 path (M = 2..4 rows past att_par)
                                        run each layer's o, gate/up, down and the next qkv projection
                                        with their norms in one persistent kernel (1), or as one
                                        kernel per step (0, the default: measured faster) */
  int prefill_tc;                    /* prefill the prompt's full blocks with the tensor-core W4A8
                                        GEMM (tcgen05) over up to 2,048 rows at a time (1: attention
                                        with one query row of a head per block, measured fastest; 3:
                                        4 rows of a head per block; 2: 4 heads of a row per block), or
                                        block by block through the GEMV path (0); same values in all
                                        four */
  int slots;                         /* ENGINE_SLOTS (1): conversations kept for the prefix cache (the
                                        active one and slots - 1 stored, each with its own K/V) */
  int slot_min_reuse;                /* ENGINE_SLOT_MIN_REUSE (32) */
  int kv_owners;                     /* KV sharing (owner_of, gemma4_engine.cpp:1251; the E2B model: 15):
                                        layers [0, kv_owners) own a KV cache, every later layer reads
                                        the cache of the last owner of its type (sliding or global)
                                        and has no k/v projections; 0 (the default) = every layer
                                        owns its cache */
  int mlp_shared;                    /* MLP width of the KV-shared layers (the E2B model: 12,288, twice
                                        the owners' 6,144); 0 = mlp */
  int ple;                           /* per-layer embeddings (the E2B model's PLE, gemma4_engine.cpp:1270-1288,
                                        1379-1388): 256 inputs per layer from a [vocab][n_layers x 256]
                                        table and a projection of the embedding, gated into the residual
                                        stream after each layer's MLP (1), or none (0, the default); needs
                                        prefill_int8 = decode_int8 = 1 (the reference's int8 branch) */
} g4_engine_config;
typedef struct {
  int rounds, ngram_rounds, drafted, accepted, prefill_tokens, decode_tokens;
  double prefill_ms, decode_ms; /* host wall clock */
  double decode_gpu_ms;         /* CUDA events on the engine stream around the decode calls */
  int verify_passes, verify_rows, draft_steps;
  double verify_gpu_ms, draft_gpu_ms; /* CUDA events around each verify pass / each round's drafts */
  long long h2d_bytes, d2h_bytes;     /* host<->device copies made by the decode calls */
  long long kernel_launches;          /* kernels the decode calls ran (graph kernel nodes included) */
  int head_fallbacks;                 /* verify passes that read the full exact head: the certified
                                         screen kept more than screen_lim rows, or was skipped */
  int screen_skipped;                 /* verify passes that skipped the screen (head_screen = 2) */
  int ngram_accepted;                 /* drafts accepted in prompt-lookup rounds */
} g4_engine_stats;

int g4_engine_default_config(g4_engine_config* cfg);
/* Allocates the weights (generated on the device from cfg->seed), KV cache and buffers. */
int g4_engine_create(const g4_engine_config* cfg, g4_engine** out);
void g4_engine_destroy(g4_engine* e);
/* An engine for another independent request stream over the weights of `weights` (same model
 * dimensions and seed; ctx_max at most the weights engine's): its own KV cache, activations, round
 * state, CUDA stream and graphs, no copy of the weights.  `weights` must outlive it.  Independent
 * streams (the reference serves one request at a time) run concurrently through
 * g4_engine_decode_async. */
int g4_engine_create_shared(const g4_engine_config* cfg, const g4_engine* weights, g4_engine** out);
/* ---------------------------------------------------------------- checkpoints
 * A checkpoint in the reference's format, read on the host (no GPU needed): <ckpt>/model.safetensors
 * (path may name the file or the directory), found through the reference's index file (one line per
 * tensor: name, dtype, absolute offset, byte count, comma-separated shape, as tools/make_index.py
 * writes it and gemma4_engine.cpp:1216-1217 reads it) or, when index is NULL, through the
 * safetensors header itself.  The file is mapped read-only; every tensor's extent and byte count
 * (dtype x shape) are checked at open. */
typedef struct g4_checkpoint g4_checkpoint;
int g4_checkpoint_open(const char* path, const char* index, g4_checkpoint** out);
void g4_checkpoint_close(g4_checkpoint* ck);
/* Number of tensors, and one tensor's dtype ("BF16", "I32", ...), shape (up to shape_cap dims) and
 * byte count. */
int g4_checkpoint_count(const g4_checkpoint* ck);
int g4_checkpoint_tensor(const g4_checkpoint* ck, const char* name, char* dtype, int dtype_cap, long long* shape,
                         int shape_cap, int* ndim, long long* nbytes);
/* The target model the checkpoint holds: hidden, n_layers, mlp and vocab are written into cfg (its
 * other fields are left as they are) after every tensor the engine reads has been checked (the
 * reference's names, gemma4_engine.cpp:1222-1231: layers.<l>.self_attn.{q,k,v,o}_proj and
 * mlp.{gate,up,down}_proj as weight_packed I32 [N][K/8] (or U8 [N][K/2]) + weight_scale BF16
 * [N][K/32], the layer's norms BF16, layer_scalar BF16 (1 when absent), norm.weight,
 * embed_tokens.weight BF16 [vocab][hidden]).  Trailing layers without k/v projections (and k_norm)
 * are KV-shared: cfg->kv_owners is set to the first of them, and cfg->mlp_shared to their MLP width
 * when it differs from the owners'; per-layer embeddings (embed_tokens_per_layer,
 * per_layer_model_projection, per_layer_projection_norm and each layer's per_layer_input_gate,
 * per_layer_projection, post_per_layer_input_norm) set cfg->ple.  Parts of the real E2B model this
 * build does not run (head_dim other than 256, MLP widths that vary otherwise) give
 * G4_ERR_UNSUPPORTED with the part named. */
int g4_checkpoint_config(const g4_checkpoint* ck, g4_engine_config* cfg);
/* An engine whose target weights are the checkpoint's (the reference's q4 / bfvec loading,
 * gemma4_engine.cpp:172-175, 1222-1231): cfg's model sizes are replaced by the checkpoint's
 * (g4_checkpoint_config); the MTP drafter, when cfg->drafter is set, is generated from cfg->seed
 * (the reference reads its drafter from a separate checkpoint of another format).  ck may be
 * closed once this returns.  A checkpoint with per-layer embeddings is refused (G4_ERR_UNSUPPORTED):
 * that path is not verified against the oracle in this build. */
int g4_engine_create_from_checkpoint(const g4_engine_config* cfg, const g4_checkpoint* ck, g4_engine** out);
/* One target forward (fwd) over M <= 32 host tokens at positions pos0..; int8 selects the W4A8
 * path for M >= 2.  When want, rows hf.. get the greedy next token G (host [M]) and, if hbuf is
 * non-null, the final-normed hidden (host [M][hidden]). */
int g4_engine_forward(g4_engine* e, const int32_t* toks, int M, int pos0, int want, int hf, int int8, int32_t* G,
                      float* hbuf);
/* One MTP draft step: token, hidden h (host [hidden]), query position, last target position P. */
int g4_engine_draft(g4_engine* e, int32_t tok, const float* h, int pos, int P, int32_t* out_tok, float* h_next);
/* ENGINE_FAKE_CTX (gemma4_engine.cpp:1249-1250): fill positions [0, n) of every layer's K and V
 * with the reference's seeded LCG values (K then V per element, one stream over the layers); the
 * next prefill then starts at position n.  n = 0 turns it off. */
int g4_engine_fake_ctx(g4_engine* e, int n);
/* Prefill a prompt (host [n]) in blocks of prefill_block and reset the decode state; *first_token =
 * the greedy token after the prompt. */
int g4_engine_prefill(g4_engine* e, const int32_t* prompt, int n, int32_t* first_token);
/* Prefill from prompt position start (0 <= start < n), keeping the K/V of positions < start: the
 * caller guarantees that they hold prompt[0, start) (an earlier request's prefix; the request API
 * below tracks it).  The prefill blocks start at start, as run_req's do after a prefix-cache hit
 * (gemma4_engine.cpp:1597-1600), so the values are those of the reference's reuse, not of a full
 * prefill.  start = 0 is g4_engine_prefill. */
int g4_engine_prefill_from(g4_engine* e, const int32_t* prompt, int n, int start, int32_t* first_token);
/* Continue speculative greedy decode for up to max_rounds rounds or max_tokens committed tokens
 * (whichever comes first) or a stop token; out host [max_tokens] (may be NULL), *n_out = tokens
 * committed by this call; stats (may be NULL) accumulate since the prefill.
 * Prompt lookup, the choice between it and the MTP drafts, greedy acceptance and the commit run on
 * the device (the spec loop of run_req, gemma4_engine.cpp:1616-1663).  Once every verify row
 * takes the split-KV path (position > att_par) and graphs are on, all rounds of the call are one
 * graph launch (a conditional WHILE over rounds, IF for the drafts, SWITCH over the verify rows)
 * followed by one copy of the committed tokens; verify_gpu_ms and draft_gpu_ms then come from
 * %globaltimer stamps taken by the round kernels, decode_gpu_ms from CUDA events around the call. */
int g4_engine_decode(g4_engine* e, int max_rounds, int max_tokens, int32_t* out, int* n_out, g4_engine_stats* stats);
/* g4_engine_decode in two halves, so that several engines decode at the same time: _async enqueues
 * the call's rounds (one launch of the round-loop graph; needs graphs on and a position past
 * att_par) on the engine's stream, after start_event (a cudaEvent_t, may be NULL) when given, and
 * returns; _wait completes it (out, n_out, stats as for g4_engine_decode; ms_since_start, may be
 * NULL, = device time from start_event to the end of the rounds). */
int g4_engine_decode_async(g4_engine* e, int max_rounds, int max_tokens, void* start_event);
int g4_engine_decode_wait(g4_engine* e, int32_t* out, int* n_out, g4_engine_stats* stats, void* start_event,
                          float* ms_since_start);
/* One request of run_req (gemma4_engine.cpp:1581-1613) with its prefix cache (:1569-1594): the
 * conversation (the active one or a stored slot) whose committed tokens share the longest prefix
 * with the prompt becomes active (a stored one is swapped in); if no stored conversation shares
 * more than the active one and the best shares fewer than slot_min_reuse tokens, the least recently
 * used slot takes the active conversation and the request starts from an empty cache.  Then prefill
 * from min(shared, n - 1) (g4_engine_prefill_from) and decode until max_new tokens (the first from
 * the prefill) or a stop token.  out host [max_new]; *n_out = tokens, cut after the first stop
 * token.  max_new = 0 prefills only (the prompt becomes the conversation; out may be NULL).  With
 * slots = 1 only the active conversation is reused.  on_tokens may be NULL. */
typedef struct {
  int prompt_tokens;                 /* n */
  int reused;                        /* prompt positions whose K/V came from the cache */
  int slot;                          /* 0: the active conversation; i: stored slot i - 1 was switched in
                                        or, on an eviction, took the active conversation */
  int tokens;                        /* *n_out */
  double prefill_ms, decode_ms;      /* host wall clock */
  int slot_switches, slot_evictions; /* totals since the engine was created */
  int kv_len;                        /* positions of the active conversation now in the cache */
  int rounds, ngram_rounds, ngram_accepted; /* decode rounds of this request, those that used prompt
                                               lookup, drafts they accepted */
} g4_request_info;
/* Drafts per round k (0..3; the reference's BENCH_MODE, gemma4_engine.cpp:1682): takes effect at the
 * next decode call. */
int g4_engine_set_k_draft(g4_engine* e, int k);
/* Called by g4_engine_request with tokens as they commit: the first token after the prefill, then
 * each decode round's tokens (the request then decodes one round per g4_engine_decode call). */
typedef void (*g4_token_cb)(const int32_t* tokens, int n, void* user);
int g4_engine_request(g4_engine* e, const int32_t* prompt, int n, int max_new, int32_t* out, int* n_out,
                      g4_request_info* info, g4_token_cb on_tokens, void* user);
/* Per-round records since the prefill, 6 ints each: {drafts verified nd, prompt lookup used (1) or MTP
 * (0), the MTP drafts (-1 padded), accepted nacc}; out host [cap_rounds][6]; *n_rounds = rounds
 * recorded (records past the engine's capacity of ctx_max rounds are not kept). */
int g4_engine_trace(g4_engine* e, int32_t* out, int cap_rounds, int* n_rounds);
/* Device time of one verify pass of M rows at the current position: the captured pass replayed reps
 * times between CUDA events on the engine stream (what a round's verify costs, for roofline
 * accounting).  Needs graphs on and a position past att_par. */
int g4_engine_time_verify(g4_engine* e, int M, int reps, double* ms_per_pass);
/* Profiling aid: %globaltimer stamps (ns) of the stage boundaries inside the persistent segment
 * kernels of the most recent fused verify pass, [n_layers + 2 launches][first CTA, last CTA][24]
 * (0 = start, 1 = after the wait on the previous kernel, 2-15 = after each stage and barrier,
 * 20/22 = weight streamer start/end); *n = the element count. */
int g4_engine_seg_trace(g4_engine* e, unsigned long long* out, int cap, int* n);
/* Continue src's stream in dst (same model dimensions): the KV rows of every layer up to src's
 * position, the history, the last hidden state and the round state are copied (device to device). */
int g4_engine_copy_state(g4_engine* dst, const g4_engine* src);
/* Decode state after a prefill or decode call: K and V rows of positions [0, npos) of every layer
 * (host [n_layers][npos][256] bf16 each, may be NULL), the committed history (host seq [seq_cap]
 * may be NULL, *seq_len its length), the final-normed hidden of the last committed row (host
 * [hidden], may be NULL) and its position *P. */
int g4_engine_export_state(g4_engine* e, int npos, uint16_t* Kc, uint16_t* Vc, int32_t* seq, int seq_cap, int* seq_len,
                           float* hprev, int* P);
/* Per-phase device time (CUDA events on the engine stream) while profiling is on: out_ms[6] =
 * embed+norms+RoPE+residual, linears, attention, head, drafter, copies; out_marks[6] = intervals.
 * enable = 1 starts (and clears), 0 stops, -1 only reads.  Outputs may be NULL. */
int g4_engine_phase_times(g4_engine* e, int enable, double* out_ms, long long* out_marks);
/* run_req: prefill the prompt, then speculative greedy decode until n_new tokens (the first from
 * the prefill) or a stop token (1 or 106).  out host [n_new]. */
int g4_engine_generate(g4_engine* e, const int32_t* prompt, int n, int n_new, int32_t* out, int* n_out,
                       g4_engine_stats* stats);

#ifdef __cplusplus
}
#endif
#endif
