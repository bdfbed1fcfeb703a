/*
 * ojx.h — C-ABI of libojx.so, the B200 (sm_100a) runtime and GEMM engine that
 * backs the `torchcl` Python package (torchcl.matmul / torchcl.blas.gemm and the
 * lazily fused elementwise epilogue).
 *
 * Every function returns an int status (OJX_OK == 0).  On failure a
 * thread-local message is available from ojx_last_error().  All pointers are
 * plain device (or host) addresses; no PyTorch types cross this boundary.
 *
 * Each declaration names the reference interface it replaces (path:line inside
 * the OjasX project).  The reference implements these in Python over pyopencl;
 * here they are native C++/CUDA.
 */
#ifndef OJX_H_
#define OJX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OJX_ABI_VERSION 1

/* ── status codes ─────────────────────────────────────────────────────────
 * OJX_ERR_INVALID  -> ValueError   (torchcl/api.py:433-439 raises on bad shapes)
 * OJX_ERR_OOM      -> MemoryError  (after evict-and-retry, torchcl/runtime/memory.py:109-115)
 * OJX_ERR_TIMEOUT  -> RuntimeError (a bounded device-side wait expired; the kernel returned)
 * OJX_ERR_CUDA     -> RuntimeError (any CUDA runtime/driver failure)
 * OJX_ERR_BOUNDS   -> RuntimeError (bounds-checking build only: a device-side check failed)
 */
enum {
  OJX_OK = 0,
  OJX_ERR_INVALID = 1,
  OJX_ERR_OOM = 2,
  OJX_ERR_CUDA = 3,
  OJX_ERR_TIMEOUT = 4,
  OJX_ERR_UNSUPPORTED = 5,
  OJX_ERR_NOT_INITIALIZED = 6,
  OJX_ERR_BOUNDS = 7
};

/* element types */
enum { OJX_F32 = 0, OJX_BF16 = 1, OJX_F16 = 2 };

/* unary epilogue ops; the set and formulas of torchcl/jit/compiler.py:33-45 */
enum {
  OJX_UN_NONE = 0,
  OJX_UN_RELU = 1,
  OJX_UN_SIGMOID = 2,
  OJX_UN_TANH = 3,
  OJX_UN_NEG = 4,
  OJX_UN_ABS = 5,
  OJX_UN_EXP = 6,
  OJX_UN_LOG = 7,
  OJX_UN_SQRT = 8,
  OJX_UN_SILU = 9,
  OJX_UN_GELU = 10, /* tanh approximation, torchcl/jit/compiler.py:43 */
  OJX_UN_SQUARE = 11
};

/* binary epilogue ops; torchcl/jit/compiler.py:47-52 */
enum { OJX_BIN_NONE = 0, OJX_BIN_ADD = 1, OJX_BIN_SUB = 2, OJX_BIN_MUL = 3, OJX_BIN_DIV = 4 };

/* shape of the epilogue's second operand */
enum {
  OJX_OPERAND_NONE = 0,
  OJX_OPERAND_ROW = 1,  /* bias[N], broadcast over rows (matmul.cl:218 `bias[out_col + j]`) */
  OJX_OPERAND_FULL = 2  /* X[M,N] with leading dimension ld_operand (fused binary of api.py:109-128) */
};

/* how an fp32 GEMM is computed */
enum {
  OJX_FP32_AUTO = 0,   /* 3xTF32 on tcgen05 when the shape allows, FFMA otherwise */
  OJX_FP32_3XTF32 = 1, /* split x = hi + lo (both tf32), C = Ah*Bh + Ah*Bl + Al*Bh, fp32 accumulate */
  OJX_FP32_FFMA = 2    /* SIMT fp32 FMA, k ascending per output element */
};

#define OJX_MAX_UNARY 8
#define OJX_MAX_PEERS 8        /* ranks an all-gathering GEMM can write to */
#define OJX_IPC_HANDLE_BYTES 64

/* One GEMM with its fused epilogue:
 *   acc[m,n] = sum_k op(A)[m,k] * op(B)[k,n]              (fp32 accumulate)
 *   v        = operand_kind ? bin(acc, X) : acc           (bin(X, acc) if operand_is_lhs)
 *   v        = unary[n_unary-1](...unary[0](v))
 *   C[m,n]   = convert(v, dtype_c)
 * op(A) = A (row-major [M,K], lda) or A^T (A stored row-major [K,M]) when trans_a.
 * op(B) = B (row-major [K,N], ldb) or B^T (B stored row-major [N,K]) when trans_b.
 * Replaces OpenCLEngine.run_matmul / run_matmul_bias / run_linear / run_matmul_fp16
 * (torchcl/ops/engine.py:156-255, 351-392) plus the JIT's second launch
 * (torchcl/jit/compiler.py:99-133): one launch, one store.
 */
typedef struct ojx_gemm_desc {
  int64_t M, N, K;
  int32_t dtype_a, dtype_b, dtype_c, dtype_operand; /* OJX_F32 / OJX_BF16 / OJX_F16 */
  int32_t trans_a, trans_b;
  int64_t lda, ldb, ldc, ld_operand; /* leading dimensions in elements; 0 = dense */
  const void* a;
  const void* b;
  void* c;
  const void* operand; /* bias[N] or X[M,N]; may be NULL when operand_kind == NONE */
  int32_t operand_kind; /* OJX_OPERAND_* */
  int32_t binary_op;    /* OJX_BIN_*; ADD when a bias is given */
  int32_t operand_is_lhs; /* 1: v = bin(X, acc) (e.g. sub(X, matmul(A,B))) */
  int32_t n_unary;
  int32_t unary[OJX_MAX_UNARY];
  int32_t fp32_mode; /* OJX_FP32_* */
  int32_t flags;     /* OJX_GEMM_FLAG_* */
} ojx_gemm_desc;

/* route selection overrides (tests and benchmarks) */
#define OJX_GEMM_FLAG_FORCE_SIMT 0x1   /* SIMT kernel for any dtype */
#define OJX_GEMM_FLAG_NO_SKINNY 0x2    /* never take the split-K skinny route */
#define OJX_GEMM_FLAG_FORCE_SKINNY 0x4 /* skinny route when M <= 16 even if a tile kernel would fit */
#define OJX_GEMM_FLAG_PAIR 0x8         /* CTA-pair tiles (cta_group::2, 256 x 256) where they apply:
                                          ~2 % faster in short runs, slower under the power cap */
#define OJX_GEMM_FLAG_SKINNY_COUNTER 0x10 /* skinny route: hand split-K partials over through the
                                             arrival counter even where the tagged hand-off applies
                                             (same sums, same result bits) */

/* Which kernel family ojx_gemm used for its most recent call on this thread. */
enum {
  OJX_ROUTE_NONE = 0,
  OJX_ROUTE_TC_F16 = 1,   /* tcgen05 kind::f16 tile GEMM (bf16/fp16) */
  OJX_ROUTE_TC_3XTF32 = 2,/* tcgen05 kind::tf32, three MMAs per k-step */
  OJX_ROUTE_SKINNY = 3,   /* tcgen05 swap-AB stream-K skinny GEMM */
  OJX_ROUTE_SIMT = 4,     /* SIMT FMA GEMM (any shape, any stride) */
  OJX_ROUTE_FLASH_ATTN = 5 /* ojx_attention: fused tcgen05 attention kernel */
};

typedef struct ojx_device_info {
  char name[256];
  int32_t device;
  int32_t cc_major, cc_minor;
  int32_t sm_count;
  int64_t total_mem_bytes;
  int64_t l2_bytes;
  int32_t max_smem_per_block;
  int32_t clock_khz;
} ojx_device_info;

typedef struct ojx_pool_stats {
  int64_t alloc_count;            /* fresh cudaMalloc calls */
  int64_t reuse_count;            /* requests served from a cached block */
  int64_t free_count;
  int64_t active_bytes;           /* capacity of blocks handed out */
  int64_t cached_bytes;           /* capacity of blocks parked in bins */
  int64_t peak_bytes;
  int64_t total_allocated_bytes;  /* sum of all cudaMalloc sizes */
  int64_t active_buffers;
  int64_t evictions;              /* evict-and-retry events after an OOM */
} ojx_pool_stats;

/* Streams are plain cudaStream_t values; NULL is the legacy default stream. */
typedef void* ojx_stream;
typedef void* ojx_event;

/* ── runtime (replaces torchcl/runtime/context.py:26-146) ─────────────── */
int ojx_abi_version(void);
int ojx_device_count(int* count);                       /* context.py:131-140 is_available */
int ojx_init(int device, ojx_device_info* info);        /* context.py:26-100 init_opencl, 169-186 */
int ojx_current_device(int* device);
int ojx_synchronize(void);                               /* context.py:143-146 synchronize */
const char* ojx_last_error(void);                        /* thread-local message of the last failure */
int ojx_poll_device_error(void);                         /* reads and clears the kernels' error word */
/* 1 in the bounds-checking build (libojx_debug.so, compiled with OJX_DEBUG_BOUNDS), else 0.
 * That build checks every TMA tile origin and epilogue store of the GEMM and attention
 * kernels on the device; a failed check skips the access, and the next
 * ojx_poll_device_error returns OJX_ERR_BOUNDS with the site and coordinates.  No
 * counterpart in the reference (which has no device-side checks); it serves the
 * sanitizer role of compute-sanitizer, which this library's tests do not rely on. */
int ojx_debug_bounds_enabled(void);
int ojx_set_wait_budget(uint64_t cycles);                /* bound of every device-side spin wait */
uint64_t ojx_kernel_launch_count(void);                  /* kernels this library launched so far */
int ojx_last_route(void);                                /* OJX_ROUTE_* of this thread's last ojx_gemm */

/* ── caching allocator (replaces torchcl/runtime/memory.py:61-203 CLBufferPool) ── */
int ojx_malloc(size_t nbytes, void** dptr, size_t* capacity); /* memory.py:85-127 allocate */
int ojx_free(void* dptr);                                      /* memory.py:129-137 free */
int ojx_empty_cache(void);                                     /* memory.py:139-143 */
int ojx_pool_stats_get(ojx_pool_stats* out);                   /* memory.py:198-203 get_stats */
int ojx_pool_bin_size(size_t nbytes, size_t* capacity);        /* memory.py:20-24 _next_power_of_two */
int ojx_pool_debug_fail_next(int64_t n_allocs);                /* test hook: the next n cudaMalloc calls fail */

/* ── copies (memory.py:145-196) ───────────────────────────────────────── */
int ojx_memcpy_h2d(void* dst, const void* src, size_t nbytes, ojx_stream s);
int ojx_memcpy_d2h(void* dst, const void* src, size_t nbytes, ojx_stream s);
int ojx_memcpy_d2d(void* dst, const void* src, size_t nbytes, ojx_stream s);
int ojx_memset(void* dst, int value, size_t nbytes, ojx_stream s); /* memory.py:192-196 zero_fill */
int ojx_host_alloc(size_t nbytes, void** host_ptr);                 /* pinned host memory */
int ojx_host_free(void* host_ptr);

/* ── streams and events (replaces torchcl/runtime/stream.py:32-132) ───── */
int ojx_stream_create(ojx_stream* s);
int ojx_stream_destroy(ojx_stream s);
int ojx_stream_synchronize(ojx_stream s);
int ojx_stream_wait_event(ojx_stream s, ojx_event e);
int ojx_event_create(ojx_event* e, int enable_timing);
int ojx_event_destroy(ojx_event e);
int ojx_event_record(ojx_event e, ojx_stream s);
int ojx_event_query(ojx_event e, int* done);
int ojx_event_synchronize(ojx_event e);
int ojx_event_elapsed_ms(ojx_event start, ojx_event end, float* ms);

/* ── compute ──────────────────────────────────────────────────────────── */
/* GEMM + fused epilogue.  Replaces engine.py:156-255 and 351-392 and
 * the matmul.cl kernels matmul_reg_tiled_f32 (19-120), matmul_reg_tiled_bias_f32
 * (123-224), linear_forward_tiled_f32 (297-343), matmul_naive_f32 (346-364),
 * matmul_bias_f32 (366-385), matmul_tiled_fp16 (422-463).  Asynchronous on s. */
int ojx_gemm(const ojx_gemm_desc* d, ojx_stream s);

/* Elementwise fusion: out[i] = u_n(...u_1(bin(a[i], b[i]))) over a flat range.
 * b == NULL -> unary chain only.  Replaces JITCompiler.fuse_elementwise_chain and
 * fuse_binary_then_unary (torchcl/jit/compiler.py:64-133). */
int ojx_elementwise(void* out, int32_t dtype_out, const void* a, int32_t dtype_a,
                    const void* b, int32_t dtype_b, int32_t binary_op,
                    const int32_t* unary, int32_t n_unary, int64_t n, ojx_stream s);

/* out[cols, rows] = in[rows, cols]^T.  Replaces run_transpose (engine.py:332-349,
 * matmul.cl:387-398 transpose_f32). */
int ojx_transpose(void* out, const void* in, int64_t rows, int64_t cols, int32_t dtype, ojx_stream s);

/* out[i] = value.  Replaces run_fill (engine.py run_fill, elementwise.cl fill_f32). */
int ojx_fill(void* out, double value, int64_t n, int32_t dtype, ojx_stream s);

/* dtype conversion.  Replaces AdaptivePrecision pack/unpack (torchcl/liquid/precision.py:68-103,
 * precision.cl:7-27). */
int ojx_cast(void* out, int32_t dtype_out, const void* in, int32_t dtype_in, int64_t n, ojx_stream s);

/* out[c] = sum over r < rows of in[r * ld + c] (ld 0 = cols), accumulated in fp32:
 * the bias gradient of a linear layer.  Replaces run_sum_columns
 * (torchcl/ops/engine.py:807-822) and its kernel sum_columns_f32
 * (torchcl/kernels/reduction.cl:170-181), called from LinearFunction.backward
 * (torchcl/autograd.py:404-408).  The reference adds the rows of a column in
 * order with one accumulator; here rows are summed in blocks of 64 (each block in
 * row order, then the block sums in block order), which is deterministic and
 * reads the input once at full bandwidth. */
int ojx_sum_columns(void* out, int32_t dtype_out, const void* in, int32_t dtype_in, int64_t rows,
                    int64_t cols, int64_t ld, ojx_stream s);

/* ── multi-GPU: W column-sharded GEMM with the output all-gathered by the GEMM
 * epilogue itself.  The reference's only "distributed" code is a host-side loop
 * (torchcl/mesh/collective.py:33-91: to_cpu, torch.cat, to_opencl); there is no
 * device-side counterpart, so these entry points are new.
 *
 * Each rank allocates its full C[M, N_total] (ojx_malloc), exports it with
 * ojx_ipc_get_handle, exchanges the 64-byte handles out of band (e.g. a
 * torch.distributed all_gather_object) and opens the peers' buffers with
 * ojx_ipc_open_handle.  ojx_gemm_allgather then computes this rank's column
 * block C[:, col_offset : col_offset + d->N] = epilogue(A @ W_shard) and stores
 * every output chunk into ALL ranks' C buffers (c_peers[i], row-major, leading
 * dimension d->ldc) over NVLink, so no separate all-gather or re-layout runs.
 * The kernel makes its stores visible system-wide before it completes; a
 * stream-ordered barrier across the ranks (one small collective) must follow
 * before any rank reads its C. */
int ojx_ipc_get_handle(void* dptr, void* handle_out);               /* 64 bytes */
int ojx_ipc_open_handle(const void* handle, void** dptr);           /* peer's buffer */
int ojx_ipc_close_handle(void* dptr);
int ojx_gemm_allgather(const ojx_gemm_desc* d, void* const* c_peers, int32_t n_peers,
                       int64_t col_offset, ojx_stream s);

/* Decode GEMM (the skinny split-K route of ojx_gemm: 1 <= M <= 16, bf16 or fp16
 * A and B, A row-major, 16-byte aligned rows) that allocates no device memory.
 * No counterpart in the reference.  For callers that may not have the library
 * call cudaMalloc: engines that reserve the GPU's memory up front and treat
 * later allocations as failures, or latency-critical loops in which an
 * allocation could synchronise the device.  Its scratch is a fixed 8 MiB array
 * that every GPU loading the library holds until exit; larger problems are
 * rejected with OJX_ERR_INVALID.  All calls share the array: calls that overlap
 * on the GPU race, so order them on one stream.  The first call on a device sets
 * the array up; make it before capturing a stream. */
int ojx_gemm_skinny_noalloc(const ojx_gemm_desc* d, ojx_stream s);

/* Batched GEMM: problem b < batch computes C_b = epilogue(op(A_b) @ op(B_b)) with
 * A_b = a + b*stride_a, B_b = b + b*stride_b, C_b = c + b*stride_c and its epilogue
 * operand at operand + b*stride_operand (strides in elements; a stride of 0 shares
 * one A, B or operand across the batch; outputs may not overlap).  bf16/fp16 and
 * 3xTF32 problems run as ONE tcgen05 launch whose tile scheduler walks every
 * problem's tiles (rank-3 TMA maps); other shapes run one launch per problem.
 * Replaces blas.bmm (torchcl/blas/__init__.py:123-150, kernel
 * matmul_batched_strided_f32 in torchcl/kernels/winograd_gemm.cl:91-119) and the
 * PrivateUse1 per-batch loop cl_bmm (torchcl/runtime/privateuse1.py:216-234). */
int ojx_gemm_batched(const ojx_gemm_desc* d, int64_t batch, int64_t stride_a, int64_t stride_b,
                     int64_t stride_c, int64_t stride_operand, ojx_stream s);

/* The GEMM with A and C in host memory (pinned, for the overlap) and B and the epilogue
 * operand on the device: the rows are processed in chunks (chunk_rows, or 0 for about
 * eight chunks of whole 128-row tile blocks); chunk i+1 uploads into dev_a, chunk i
 * computes into dev_c and chunk i-1 downloads, on three library streams, so only the
 * first upload and the last download are not hidden behind GEMM work.  dev_a ([M,K])
 * and dev_c ([M,N]) are caller-owned device buffers; A and C must be dense row-major.
 * Ordered after the work already queued on `s`; `s` waits for the last download, so
 * synchronising `s` means C is in host memory.  Replaces the upload / matmul / download
 * sequence of to_opencl + matmul + to_cpu (torchcl/api.py:210-232, 427-469), which the
 * reference runs one after another with a blocking copy on each side
 * (torchcl/runtime/memory.py:145-177). */
int ojx_gemm_host_io(const ojx_gemm_desc* d, void* dev_a, void* dev_c, int64_t chunk_rows,
                     ojx_stream s);

/* Scaled dot-product attention: for each of batch*heads problems,
 *   out = softmax(scale * Q K^T) V,  Q [M, D], K and V [N, D], out [M, D], row-major,
 * problems packed [batch][heads][rows][D].  causal: query i sees keys j <= i.  The
 * softmax divides by (sum + 1e-6) as the reference does.  max_keys > 0 keeps only the
 * first max_keys keys (2048 reproduces the reference kernel, whose score buffer
 * holds 2048 entries); 0 uses all N.  bf16/fp16 with D = 64 or 128 run ONE fused
 * kernel (tcgen05 S = QK^T and O += PV with TMEM accumulators, online softmax between
 * them; route OJX_ROUTE_FLASH_ATTN).  Otherwise, and for fp32 (3xTF32 GEMMs), two
 * batched GEMMs around a row-softmax kernel, P rounded to the input type.  Replaces
 * fused_attention / run_fused_attention (torchcl/api.py:667-695,
 * torchcl/ops/engine.py:755-773) and flash_attention.cl:8-187.  ojx_last_route
 * reports the GEMMs' route when both took the same one. */
int ojx_attention(void* out, const void* q, const void* k, const void* v, int32_t dtype,
                  int64_t batch, int64_t heads, int64_t M, int64_t N, int64_t D, float scale,
                  int32_t causal, int64_t max_keys, int32_t flags, ojx_stream s);
#define OJX_ATTN_FLAG_COMPOSED 0x1 /* GEMM + softmax + GEMM even where the fused kernel applies */
#define OJX_ATTN_FLAG_ONE_QTILE 0x2 /* fused kernel with 128 queries per CTA */
#define OJX_ATTN_FLAG_TWO_QTILE 0x4 /* fused kernel with two 128-query tiles per CTA (ping-pong;
                                       the default) */

/* ── graph capture and replay ──────────────────────────────────────────────
 * Replaces torchcl/jit/graph_runner.py: `capture_graph` (:70-86) records the
 * launches made inside a `with` block and `CapturedGraph.replay` (:58-62)
 * re-submits them.  Here the recording is a CUDA stream capture of every ojx
 * launch issued on `s` between begin and end, instantiated once into a CUDA
 * graph that one cudaGraphLaunch replays.  Launches that need scratch (the 3xTF32
 * operand split, the skinny route's partial sums and arrival counters) get
 * buffers owned by the graph, freed by ojx_graph_destroy.  `s` must be a stream
 * from ojx_stream_create (the legacy stream cannot be captured); the capture uses
 * cudaStreamCaptureModeRelaxed so the buffer pool may grow during it.  Between
 * begin and end nothing on `s` executes: synchronising `s` or reading results
 * back fails and invalidates the capture. */
typedef struct ojx_graph_s* ojx_graph;

enum { OJX_NODE_OTHER = 0, OJX_NODE_KERNEL = 1, OJX_NODE_MEMSET = 2, OJX_NODE_MEMCPY = 3 };

/* One recorded node: graph_runner.py:25-32 RecordedCommand (kernel, global and
 * local size).  `name` is the kernel's name without template arguments. */
typedef struct ojx_graph_node {
  int32_t type;
  int32_t grid[3];
  int32_t block[3];
  int32_t smem_bytes;
  char name[128];
} ojx_graph_node;

int ojx_graph_capture_begin(ojx_stream s);
/* Ends the capture on `s` and instantiates it.  On failure (e.g. the capture was
 * invalidated) the partial graph and its buffers are released. */
int ojx_graph_capture_end(ojx_stream s, ojx_graph* g);
/* Launches the whole recorded sequence on `s` (any stream of the same device). */
int ojx_graph_launch(ojx_graph g, ojx_stream s);
/* Waits for the device, then frees the graph and the buffers it owns. */
int ojx_graph_destroy(ojx_graph g);
/* Number of nodes (graph_runner.py:64-65 __len__ counts kernel launches: pass
 * kernels_only = 1 for that count). */
int ojx_graph_node_count(ojx_graph g, int kernels_only, int32_t* n);
/* Node `index` (0-based, in execution order). */
int ojx_graph_node_get(ojx_graph g, int32_t index, ojx_graph_node* out);

/* Test hook: the next ojx_gemm on a tcgen05 route runs with its TMA producer
 * silenced, so the MMA warp's bounded wait must expire and the kernel must
 * return with OJX_ERR_TIMEOUT recorded (read it with ojx_poll_device_error). */
int ojx_debug_silence_producer_once(void);

/* Test hook: in the next skinny launch that uses the tagged split-K hand-off, the
 * contributing CTAs publish no partials, so every finishing CTA's bounded poll must
 * expire; the launch returns with OJX_ERR_TIMEOUT recorded (ojx_poll_device_error)
 * and the context stays usable. */
int ojx_debug_silence_skinny_contributors_once(void);

#ifdef __cplusplus
}
#endif

#endif /* OJX_H_ */
