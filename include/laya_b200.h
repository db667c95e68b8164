/* laya_b200 — C ABI of the B200 (sm_100a) execution library for Laya decision models.
 *
 * This library is the device half of the Laya encoder + decision-head forward pass.  It
 * replaces, in the reference project (laya-cuda):
 *   - laya_cuda/runtime.py:136-197  Runtime: weight residency, shape classes, CUDA-graph LRU
 *   - laya_cuda/runtime.py:28-133   Slot: packed inputs, activations, encoder schedule, graphs
 *   - laya_cuda/laya.py:195-245     Laya.allocate_head / read_outputs / forward_head
 *   - laya_cuda/ops.py:20-71        Ops: NVRTC kernels + cuBLAS GemmEx
 *   - laya_cuda/kernels.cu:1-183    every device kernel
 * Python keeps the request contract (tokenisation, packing order, decoding) and calls this
 * library through ctypes.  Plain C types only; every function returns 0 on success or a
 * LAYA_ERR_* code, with a message available from laya_last_error().
 *
 * Threading: one engine handle per host thread at a time (the reference's Engine is not
 * thread-safe either, docs/guide.md:17).  Different handles may run concurrently, e.g. one
 * host thread per GPU.
 */
#ifndef LAYA_B200_H
#define LAYA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LAYA_OK 0
#define LAYA_ERR_INVALID 1     /* bad argument, configuration, tensor name or shape -> ValueError */
#define LAYA_ERR_CUDA 2        /* CUDA runtime/driver failure                       -> RuntimeError */
#define LAYA_ERR_DEVICE 3      /* a kernel reported an error (bad index, pipeline wait timeout) */
#define LAYA_ERR_STATE 4       /* call in the wrong state (not finalised, closed)   -> RuntimeError */
#define LAYA_ERR_NO_DEVICE 5   /* no usable sm_100 device                           -> RuntimeError */

#define LAYA_DTYPE_F32 0
#define LAYA_DTYPE_F16 1
#define LAYA_DTYPE_BF16 2

#define LAYA_PRECISION_BF16 0  /* 16-bit GEMM/attention operands: bfloat16 (fp32 accumulate) */
#define LAYA_PRECISION_F16 1   /* 16-bit operands: float16, as the reference (runtime.py:157-158) */

/* Model geometry, from encoder/config.json and rl_agent_config.json (laya.py:55-99). */
typedef struct laya_config {
  int32_t vocab;            /* encoder vocab_size */
  int32_t width;            /* hidden_size, a multiple of 64, <= 1024 */
  int32_t heads;            /* num_attention_heads; width / heads must be 64 */
  int32_t layers;           /* num_hidden_layers */
  int32_t intermediate;     /* intermediate_size F (GeGLU: Wi is 2F x width) */
  int32_t global_every;     /* global_attn_every_n_layers */
  int32_t window;           /* local_attention // 2 (keys within +-window) */
  float theta_global;       /* RoPE theta of full-attention layers */
  float theta_local;        /* RoPE theta of sliding-window layers */
  float eps;                /* encoder norm_eps */
  int32_t max_len;          /* rl_agent_config max_len (<= 1024) */
  int32_t head_layers;      /* decision-head transformer layers (>= 1) */
  int32_t n_act;            /* action-head outputs: len(act_costs) + 1 */
  int32_t precision;        /* LAYA_PRECISION_* */
} laya_config;

typedef struct laya_metrics {
  float gpu_ms;             /* CUDA-event time of the forward pass (graph or eager) */
  int32_t rows;             /* shape class: packed token rows */
  int32_t batch;            /* shape class: questions (power of two) */
  int32_t options;          /* shape class: options (power of two >= 8) */
  int32_t cache_miss;       /* the shape class had no cached slot */
  int32_t graph_capture;    /* this call captured the class's CUDA graph */
  int32_t graph_replay;     /* this call ran a captured graph */
  int32_t kernel_launches;  /* kernels launched by this forward pass */
  uint64_t owned_gpu_bytes; /* device bytes held by the engine after the call */
} laya_metrics;

typedef struct laya_engine laya_engine;

/* Replaces Runtime.__init__ (runtime.py:137-146): selects `device`, creates the stream.
 * max_cached_shapes bounds the shape-class LRU (engine.py:12-13: 1..64). */
int laya_create(const laya_config* cfg, int device, int max_cached_shapes, laya_engine** out);

/* Replaces the per-tensor validation and upload of runtime.py:147-158.  `name` must be one of
 * Laya.weight_shapes() (laya.py:167-190) and `shape` must match it exactly; "temperature" is
 * accepted and ignored, as the reference does.  `host` holds the values in `dtype`. */
int laya_load_tensor(laya_engine* e, const char* name, int dtype, const int64_t* shape, int ndim,
                     const void* host);

/* Replaces the whole weight load of runtime.py:147-158 (safetensors read, name and shape checks,
 * per-tensor upload): reads the safetensors file at `path` (F32, F16 or BF16 tensors), checks
 * that its tensor names are exactly Laya.weight_shapes() ("Checkpoint tensor names do not match
 * the Laya adapter") and every shape ("Incompatible tensor shape: <name>"), both
 * LAYA_ERR_INVALID, and places every tensor in one device allocation.  The file is memory-mapped
 * and streamed through pinned staging chunks copied by several host threads; uploads are
 * asynchronous and the conversion to the stored type (16-bit GEMM operands in the engine's
 * precision, fp32 for norms, biases, embeddings and the head tail) and the GeGLU row interleave
 * run on the device.  Replaces any tensors loaded before; call laya_finalize afterwards. */
int laya_load_checkpoint(laya_engine* e, const char* path);

/* Host only: parses the safetensors header at `path` and checks every tensor's byte range
 * against the file, as laya_load_checkpoint does before uploading; returns the tensor count and
 * their total element count.  LAYA_ERR_INVALID for a malformed or truncated file. */
int laya_scan_checkpoint(const char* path, int64_t* tensors, int64_t* elements);

/* After all tensors are loaded: checks completeness and builds the RoPE tables
 * (runtime.py:159-165) and the device-side weight layouts. */
int laya_finalize(laya_engine* e);

/* Replaces Runtime.predict (runtime.py:171-186) + Slot.fill/run (runtime.py:52-68, 115-133) +
 * Laya.read_outputs (laya.py:206-208).  Items are the adapter's (ids, markers, kind) triples
 * flattened: tokens = concat(ids), lengths[i] = len(ids_i), markers = concat(markers),
 * marker_counts[i] = len(markers_i), kinds[i] = question type.  The call packs the rows,
 * uploads them, runs the class's CUDA graph (capturing it on first use) or the eager pass,
 * and writes logits_out[i * options + j] (option logits, fp32, options = the class's option
 * count reported in metrics->options; the caller sizes the buffer with laya_shape_class) and
 * acts_out[i * n_act + a].  capture: 0 eager pass, 1 CUDA graph of the class (captured on first
 * use, kept in the LRU), 2 auto: graph for classes of at most 8192 packed rows, eager above. */
int laya_predict(laya_engine* e, const int32_t* tokens, const int32_t* lengths, const int32_t* markers,
                 const int32_t* marker_counts, const int32_t* kinds, int n_items, int capture,
                 float* logits_out, float* acts_out, laya_metrics* metrics);

/* laya_predict in two halves, so a host can pack and launch the next batch while the previous
 * one runs (no counterpart in the reference, whose Runtime.predict is synchronous).
 * laya_submit packs and uploads the items and enqueues the forward pass and the read-back on the
 * engine stream; it returns at once with a ticket.  At most two passes may be in flight
 * (LAYA_ERR_STATE otherwise).  laya_collect waits for the ticket's pass and writes its outputs
 * exactly as laya_predict does; tickets may be collected in any order.  The item arrays are
 * consumed by laya_submit. */
int laya_submit(laya_engine* e, const int32_t* tokens, const int32_t* lengths, const int32_t* markers,
                const int32_t* marker_counts, const int32_t* kinds, int n_items, int capture, int64_t* ticket);
int laya_collect(laya_engine* e, int64_t ticket, float* logits_out, float* acts_out, laya_metrics* metrics);

/* Shape class of a request (runtime.py:20-25): packed rows, batch and option counts. */
int laya_shape_class(const int32_t* lengths, const int32_t* marker_counts, int n_items, int32_t* rows,
                     int32_t* batch, int32_t* options);

/* Device-resident variant for throughput runs: `packed` (device memory, laya_packed_ints()
 * int32 values laid out by laya_pack()) is copied into the class's input buffer and the
 * forward pass is enqueued on the engine's stream; outputs stay on the device
 * (logits [batch][options+1] including the CLS column, acts [batch][n_act]).  No host sync. */
int laya_forward_device(laya_engine* e, const int32_t* packed, int rows, int batch, int options,
                        int capture, float* logits_dev, float* acts_dev);

/* Host-side packing used by laya_predict, exposed for laya_forward_device callers. */
int64_t laya_packed_ints(int rows, int batch, int options);
int laya_pack(const int32_t* tokens, const int32_t* lengths, const int32_t* markers, const int32_t* marker_counts,
              const int32_t* kinds, int n_items, int pad_id, int rows, int batch, int options, int32_t* packed);

/* Grows the shared activation workspace to fit a class up front (throughput callers), so no
 * forward pass has to synchronise to grow it. */
int laya_reserve(laya_engine* e, int rows, int batch, int options);

/* The engine's CUDA stream (cudaStream_t), for callers that time laya_forward_device. */
void* laya_stream(laya_engine* e);

/* Per-kernel-family device time accumulated over forward passes run with profiling on
 * (CUDA events on the engine stream around each launch of the family; eager passes only).
 * family: 0 QKV GEMM (+RoPE), 1 attention-out GEMM (+residual), 2 FFN-up GEMM (+GeGLU),
 * 3 FFN-down GEMM (+residual), 4 decision-head GEMMs, 5 attention, 6 row kernels (embedding,
 * norms, gather), 7 head tail.  flops counts 2*M*N*K over the launched (padded) rows. */
int laya_set_profiling(laya_engine* e, int enabled);
int laya_profile_read(laya_engine* e, int family, double* total_ms, int64_t* launches, double* flops);

/* Reads a loaded tensor back as fp32 (tests; runtime.weights[name].get()). */
int laya_read_tensor(laya_engine* e, const char* name, float* out, int64_t count);

/* Number of cached shape-class slots (len(runtime.slots)). */
int laya_cached_shapes(laya_engine* e, int32_t* count);

/* Device bytes owned by the engine (runtime.pool.used_bytes()/total_bytes()). */
int laya_pool_bytes(laya_engine* e, uint64_t* used, uint64_t* total);

/* Replaces Runtime.close (runtime.py:188-197).  Frees every device allocation and the handle. */
int laya_destroy(laya_engine* e);

/* Message of the last failing call on `e` (or of the last failing laya_create when e is NULL). */
const char* laya_last_error(laya_engine* e);

/* Process-wide launch options for tests of ordering and failure handling (no counterpart in the
 * reference).  programmatic_launch (1, the default, or 0): kernels of a pass launch with
 * programmatic stream serialisation, each waiting on the device for its predecessor's results.
 * wait_limit_ns: the limit of every bounded pipeline wait inside the kernels (0 restores the
 * default of 2 s); a wait that runs out makes the kernel unwind, drain what it issued and set its
 * error word, so the call reports LAYA_ERR_DEVICE.  Applies to launches made after the call;
 * CUDA graphs keep the options in effect when they were captured. */
int laya_set_launch_options(int programmatic_launch, uint64_t wait_limit_ns);

/* ------------------------------------------------------------------------------------------
 * Kernel-level entry points (device pointers, enqueued on `stream`), used by the parity tests
 * the way the reference's tests drive Ops directly (tests/test_gpu.py, tests/test_attention.py).
 * `precision` selects the 16-bit operand type (LAYA_PRECISION_*).
 * ------------------------------------------------------------------------------------------ */

/* out/residual = epilogue(x[M][K] @ w[N][K]^T).  epi: 0 store, 1 relu, 2 gelu, 3 geglu (w rows
 * pre-interleaved by laya_interleave_geglu; out is [M][N/2]), 4 qkv (RoPE when rope_tab is
 * given: 16-byte aligned fp32 [16][rope_rows][4] holding (cos f_2k, cos f_2k+1, sin f_2k,
 * sin f_2k+1) of position p at [k][p], indexed by positions[row]; q and k are written
 * [heads][M][64], v transposed [heads][64][M], all in `out`),
 * 5 residual += (fp32), 6 split-K partials ([splits][M][N] fp32 in `residual`).  bias: fp32 [N]
 * or NULL.  block_n: column tile (64, 128, 256), 0 to choose, or -128 / -256 for the CTA-pair
 * (cta_group::2, 256-row tile) kernel.  Replaces cublasGemmEx + bias/activate/layout
 * (ops.py:58-66; kernels.cu:50-82). */
int laya_op_gemm(int precision, int epi, const void* x, const void* w, int M, int N, int K, void* out, int ldo,
                 float* residual, int ldr, const float* bias, int heads, const float* rope_tab, int rope_rows,
                 const int32_t* positions, int splits, int block_n, int* err, void* stream);

/* Residual GEMM with the following LayerNorm fused (runtime.py:96-108: linear, add, layer_norm
 * of kernels.cu:20-49): residual[M][N] (fp32, row stride ldr) += x W^T + bias, then
 * out[M][N] (16-bit, row stride ldo) = LN(residual) * gamma (+ beta), population variance of the
 * centred row, eps inside the square root.  N must be 256, 512, 768 or 1024 (N/256 CTAs form a
 * cluster that owns each 128-row block); K a multiple of 64.  bias and beta may be null. */
int laya_op_gemm_ln(int precision, const void* x, const void* w, int M, int N, int K, float* residual, int ldr,
                    const float* bias, const float* gamma, const float* beta, float eps, void* out, int ldo, int* err,
                    void* stream);

/* Reorders Wi [2F][K] (gate rows then up rows) into 64-row blocks [gate_i, up_i] (host memory). */
int laya_interleave_geglu(const uint16_t* src, uint16_t* dst, int F, int K);

/* Packed attention (kernels.cu:90-154) on the tcgen05/TMEM kernel the forward pass uses.
 * qkv: q, k [heads][M][64] each, then v transposed [heads][64][M] (the layout the QKV GEMM
 * epilogue writes); out [M][heads*64].  Tiles of 128 queries from laya_attention_tiles.
 * impl 1: the forward pass's rule for splitting each tile's keys over a cluster of 2 or 4 CTAs
 * (global attention, window < 0, with M >= 384 taken as the row length, while the split grid
 * fits 4 CTAs per SM); impl 2: never split; impl 3 / 4: always split over 2 / 4 CTAs.  Unsplit
 * grids larger than the SMs' resident slots (impl 1 and 2) run the persistent kernel, whose CTAs
 * each take a list of (tile, head) items; impl 5: never split, one tile per CTA; impl 6: the
 * persistent kernel with its fewest CTAs (up to 128 items each).
 * err: device error word. */
int laya_op_attention(int precision, int impl, const void* qkv, void* out, const int32_t* tiles, int n_tiles,
                      const int32_t* starts, const int32_t* lengths, int M, int heads, int window, int* err,
                      void* stream);

/* Global attention for gathered queries only (the decision head's last layer,
 * laya.py:214-245 followed by the gather of kernels.cu:159-166): row r attends from the tokens
 * q_index[r*q_per_row .. +q_per_row) (token indices into the packed rows, duplicates allowed)
 * to every key of the row; only those rows of `out` are written.  Rows with length 0 are
 * skipped.  Layouts as laya_op_attention; tcgen05 kernel (key split as impl 1). */
int laya_op_attention_gathered(int precision, const void* qkv, void* out, const int32_t* q_index, int q_per_row,
                               const int32_t* starts, const int32_t* lengths, int n_rows, int M, int heads, int* err,
                               void* stream);

/* Builds the attention tile table (tile_q = 128) for rows packed at `starts` with
 * `lengths` into M tokens, rows longest first, then zero-fill tiles for tokens past the last
 * row, then unused slots.  Returns the number of tiles written (<= capacity) or -1. */
int laya_attention_tiles(const int32_t* starts, const int32_t* lengths, int n_rows, int M, int tile_q,
                         int32_t* tiles, int capacity);

/* residual = LN(E[ids]); x = residual (16-bit).  (kernels.cu:16-19 + runtime.py:93-95) */
int laya_op_embed_norm(int precision, const int32_t* ids, const float* table, const float* gamma, float eps, int rows,
                       int width, int vocab, float* residual, void* x, int* err, void* stream);

/* Decision-head tail (laya.py:241-245 with the features of kernels.cu:167-183), one question per
 * row of `batch`: logits[q][j] = scored[q][j] . w3 + b3 for the CLS slot and `options` option
 * slots (scored: 16-bit [batch][options+1][width]); features over the first counts[q] option
 * logits (p1, p1 - p2, entropy / log(max(c,2)), max(c,2)/255), written to features[q][4] when it
 * is not NULL; acts[q] = act_head.2(gelu(act_head.0([selected[q][0], features]))) with selected
 * fp32 [batch][options+1][width].  hidden: fp32 [batch][256] scratch; arrivals: int32 [batch],
 * zero on entry (left zero).  width a multiple of 8. */
int laya_op_head_tail(int precision, const float* selected, const void* scored, const int32_t* counts, int batch,
                      int options, int width, const float* w3, const float* b3, const float* wa0, const float* ba0,
                      const float* wa2, const float* ba2, int n_act, float* logits, float* acts, float* features,
                      float* hidden, int32_t* arrivals, void* stream);

/* residual += sum(partials[0..splits)); x = LN(residual; gamma, beta).  (kernels.cu:20-49) */
int laya_op_norm(int precision, float* residual, const float* partials, int splits, const float* gamma,
                 const float* beta, float eps, void* x, int rows, int width, void* stream);

/* ------------------------------------------------------------------------------------------
 * Allocation-free split-K residual GEMM.  No counterpart in the reference: an addition for
 * callers that cannot allocate device memory on this path, for example a serving host whose
 * own allocator owns every byte of the GPU, or a latency-critical loop where cudaMalloc /
 * cudaFree would implicitly synchronise the device and stall other streams.
 *
 *   residual[M][N] += x[M][K] @ w[N][K]^T (+ bias[N])      (same result as laya_op_gemm epi 5)
 *
 * The caller passes inputs and outputs only.  The split-K partial sums live in a static device
 * array inside the library of LAYA_STATIC_SCRATCH_FLOATS floats (16 MiB), held by every GPU that
 * loads the library until the process exits; M*N*splits must not exceed it (LAYA_ERR_INVALID
 * otherwise).  The first call on a device looks the array's device address up, so make that
 * first call before any stream capture.  All calls share the array: calls whose executions
 * overlap on the GPU (different streams, or different host threads on one device) race.  The
 * array keeps the last call's contents; every partial a call reads is written by the same call
 * first, so nothing needs clearing.  No cudaMalloc, cudaFree or allocating library routine is
 * called.  Enqueued on `stream` like the other kernel-level entry points; `stream` must belong
 * to the current device (LAYA_ERR_INVALID otherwise), whose array the call uses.  `residual` and
 * `bias` must be 16-byte aligned.  `err` (zero on entry, or NULL) receives a device error; when
 * it is set, `residual` is left unchanged. */
#define LAYA_STATIC_SCRATCH_FLOATS (4 * 1024 * 1024)
int laya_op_gemm_residual_static(int precision, const void* x, const void* w, int M, int N, int K, int splits,
                                 float* residual, const float* bias, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LAYA_B200_H */
