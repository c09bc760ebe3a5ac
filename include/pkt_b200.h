/*
 * pkt_b200 — C-ABI of the B200-native (sm_100a) persistent training megakernel.
 *
 * This is the drop-in boundary for Marco-Christiani/pkt's hot path. Plain C
 * types only (pointers, sizes, ints); device pointers are passed as void* /
 * float*, CUDA streams as void*. Every function returns an int status
 * (0 = ok, < 0 = error; pkt_last_error() gives the message) where pkt's own
 * host API returned nothing and checked no CUDA call (include/runtime.hpp:27-449).
 *
 * The C++ header include/pk/runtime.hpp wraps the runtime half of this ABI in
 * pkt's own class (pk::Runtime) so pkt programs compile unchanged against it.
 */
#ifndef PKT_B200_H
#define PKT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define PKT_OK 0
#define PKT_ERR_ARGS -1        /* bad argument / out of capacity */
#define PKT_ERR_CUDA -2        /* a CUDA runtime / driver call failed */
#define PKT_ERR_TIMEOUT -3     /* a device wait ran out of time (see pkt_runtime_status) */
#define PKT_ERR_OPCODE -4      /* device met an opcode it does not implement */
#define PKT_ERR_NCCL -5        /* an NCCL call failed */
#define PKT_ERR_UNSUPPORTED -6 /* shape / dtype / layout the kernel cannot run */

/* Device-side status word codes (pkt_runtime_status / pkt_mlp_status). */
#define PKT_DEV_OK 0
#define PKT_DEV_TIMEOUT_DEPS 1    /* controller waited too long for a dependency token */
#define PKT_DEV_TIMEOUT_PIPE 2    /* an intra-CTA pipeline wait (mbarrier) ran out */
#define PKT_DEV_BAD_OPCODE 3      /* unknown opcode in the task list */
#define PKT_DEV_BAD_ARGS 4        /* task arguments failed a device-side bounds check */

/* ---- task descriptor (byte-identical to pkt's pk::Task, include/task.cuh:22-40) */
typedef struct pkt_task_header {
  uint16_t opcode;          /* offset 0 */
  uint16_t arg_bytes;       /* offset 2 */
  uint32_t user_tag;        /* offset 4: overwritten with the task index on device */
  uint16_t buffer_read_id;  /* offset 8: dependency token waited on (0 = none) */
  uint16_t buffer_write_id; /* offset 10: token marked when the task completes (0 = none) */
  uint32_t wait_count;      /* offset 12: token count needed */
  uint32_t read_epoch;      /* offset 16: token epoch needed */
  uint32_t write_epoch;     /* offset 20: epoch published (atomic max) */
  /* offset 24: reserved[0] in pkt. Extension (0 keeps pkt semantics):
   *   bits 0-15  second token waited on, bits 16-31 second token marked. */
  uint32_t ext_ids;
  uint32_t ext_wait_count; /* offset 28: reserved[1] in pkt; count needed on the second token */
} pkt_task_header;

typedef struct pkt_task {
  pkt_task_header header;
  uint8_t args[64];
} __attribute__((aligned(16))) pkt_task;

/* Opcodes. 0-3 and 10-13 are pkt's (include/task.cuh:11-20); the rest are new. */
enum pkt_opcode {
  PKT_OP_INVALID = 0,
  PKT_OP_ZERO_MEMORY = 1,     /* pkt ZeroMemoryArgs */
  PKT_OP_AXPY = 2,            /* pkt AxpyArgs */
  PKT_OP_GEMM = 3,            /* pkt's reserved Gemm: one tcgen05 tile, pkt_gemm_tile_args */
  PKT_OP_LINEAR_FORWARD = 10, /* pkt LinearForwardArgs (fp32 SIMT tile, any shape) */
  PKT_OP_MSE_LOSS = 11,       /* pkt MSELossArgs */
  PKT_OP_LINEAR_BACKWARD = 12,/* pkt LinearBackwardArgs */
  PKT_OP_SGD_UPDATE = 13,     /* pkt SGDUpdateArgs */
  PKT_OP_BIAS_SGD = 20,       /* pkt_bias_sgd_args: reduce column partials, update bias */
  PKT_OP_LOSS_REDUCE = 21,    /* pkt_loss_reduce_args: deterministic sum of tile partials */
  PKT_OP_SGD_MIXED = 22,      /* pkt_sgd_mixed_args: fp32 master -= lr*g, bf16 shadow write */
  /* Fused data parallel (MLP grad_mode 2; peer memory between the ranks' GPUs): */
  PKT_OP_DP_WAIT = 30,        /* pkt_dp_wait_args: the next step's weights of a layer have arrived */
  PKT_OP_DP_BIAS_SEND = 31,   /* pkt_dp_bias_args: this rank's bias gradient to every rank */
  PKT_OP_DP_BIAS_APPLY = 32,  /* pkt_dp_bias_args: sum the ranks' bias gradients, SGD */
  PKT_OP_DP_REDUCE = 33       /* pkt_gemm_tile_args: an owned weight tile: sum the ranks' partials,
                                 SGD on the fp32 master, new bf16 tile to every rank */
};

/* Args of PKT_OP_GEMM: tile (tile_m, tile_n) of registered GEMM `gemm`. */
typedef struct pkt_gemm_tile_args {
  uint32_t gemm;
  uint32_t tile_m;
  uint32_t tile_n;
  uint32_t pad;
} pkt_gemm_tile_args;

typedef struct pkt_bias_sgd_args {
  const float* partials; /* [num_partials, ld] column partial sums */
  float* bias;           /* [n] updated in place (may be null: grads only) */
  float* grad_out;       /* [n] optional: the reduced gradient */
  int num_partials;
  int ld;
  int col_begin;
  int col_end;
  float lr;
  int pad;
} pkt_bias_sgd_args;

typedef struct pkt_loss_reduce_args {
  const float* partials;
  float* loss;     /* loss[0] = sum(partials) * scale, or loss[(*step)++] when step != null */
  int count;
  float scale;
  int* step;       /* optional device step counter */
} pkt_loss_reduce_args;

typedef struct pkt_sgd_mixed_args {
  const float* w;       /* fp32 master read */
  const float* g;       /* gradient */
  float* w_out;         /* fp32 master written (may equal w) */
  uint16_t* w_bf16;     /* optional bf16 copy written from the new master (may be null) */
  long long n;
  float lr;
  int pad;
} pkt_sgd_mixed_args;

/* Args of the fused data-parallel tasks. Offsets are bytes into a rank's
 * exchange region (identical layout on every rank); the region bases of all
 * ranks reach the kernel through the launch, not through the task. */
typedef struct pkt_dp_wait_args {
  int layer;
  int tiles;           /* weight tiles of the layer (each published once per CTA of a pair) */
} pkt_dp_wait_args;

typedef struct pkt_dp_bias_args {
  const float* partials; /* SEND: [num_partials, ld] column partial sums */
  float* bias;           /* APPLY: [n] updated in place */
  int num_partials;
  int ld;
  int n;
  int layer;
  int bias_off;          /* float offset of the layer in a rank's bias gradient vector */
  float lr;              /* APPLY: learning rate x gradient scale */
} pkt_dp_bias_args;

/* ---- dtypes and GEMM registration -------------------------------------- */
#define PKT_DTYPE_BF16 1
#define PKT_DTYPE_TF32 2 /* fp32 storage, TF32 tensor-core inputs */
#define PKT_DTYPE_F32 3  /* fp32 output storage */

#define PKT_MAJOR_K 0  /* operand stored [rows][K] (K contiguous) */
#define PKT_MAJOR_MN 1 /* operand stored [K][rows] (rows contiguous) */

enum pkt_epilogue {
  PKT_EPI_STORE = 0,      /* out = acc */
  PKT_EPI_BIAS_ACT = 1,   /* out = act(acc + bias) */
  PKT_EPI_MSE = 2,        /* y = acc + bias; out = dY = scale*(y - target); loss partials */
  PKT_EPI_DGRAD_RELU = 3, /* out = acc * (aux > 0) */
  PKT_EPI_WGRAD_SGD = 4,  /* w_out = w_in - lr*acc (fp32), w_bf16 = bf16(w_out) */
  PKT_EPI_WGRAD_STORE = 5, /* out = acc (fp32 gradient) */
  PKT_EPI_WGRAD_PEER = 6   /* fused data parallel (MLP grad_mode 2 only): a rank that
                              does not own the tile sends its fp32 partial to the
                              owner's exchange region; the owner sums the ranks'
                              partials, applies SGD (w_in/w_out, lr) and writes the
                              bf16 copy (w_shadow) on every rank */
};

/* One D[M,N] = sum_k A[m,k] B[n,k] problem, tiled 128 x bn. */
typedef struct pkt_gemm_desc {
  int M, N, K;
  int bn;            /* tile N: 16..256, multiple of 16 */
  int in_dtype;      /* PKT_DTYPE_BF16 or PKT_DTYPE_TF32 */
  const void* a;     /* device pointer */
  int lda;           /* elements between consecutive stored rows */
  int a_major;       /* PKT_MAJOR_K: a[m*lda+k]; PKT_MAJOR_MN: a[k*lda+m] */
  const void* b;
  int ldb;
  int b_major;
  int epilogue;      /* pkt_epilogue */
  void* out;         /* D / dY / dH / dW output */
  int ldo;
  int out_dtype;     /* PKT_DTYPE_BF16 or PKT_DTYPE_F32 */
  int relu;          /* PKT_EPI_BIAS_ACT: apply ReLU */
  const float* bias; /* [N] or null */
  const void* aux;   /* MSE: target [M,ldaux] (in_dtype storage); DGRAD: relu source H [M,ldaux] */
  int ldaux;
  float scale;       /* MSE: 2/(B*N) */
  float* loss_partials; /* MSE: [tiles_m*tiles_n] sum of squared error per tile */
  float* colsum;     /* MSE / DGRAD: [tiles_m, ldcol] per-row-block column sums of stored out */
  int ldcol;
  const float* w_in; /* WGRAD_SGD: fp32 master read (may equal w_out) [M, ldw] */
  float* w_out;      /* WGRAD_SGD: fp32 master written */
  void* w_shadow;    /* WGRAD_SGD: bf16 copy written (may be null) */
  int ldw;
  float lr;
  void* y_out;       /* MSE: optional fp32 copy of y = acc + bias */
  int ldy;
  int cta_pair;      /* 0/1: one CTA per 128 x bn tile; 2: a CTA pair per 256 x bn tile
                        (tcgen05 cta_group::2, each CTA loads its A rows and half of B);
                        must match the launch mode (pkt_runtime_set_cta_pair) */
} pkt_gemm_desc;

/* ---- runtime (pk::Runtime's C half) ------------------------------------ */
typedef struct pkt_runtime pkt_runtime;

int pkt_runtime_create(int device, pkt_runtime** out);
int pkt_runtime_destroy(pkt_runtime* rt);
/* Allocates room for max_tasks tasks (runtime.hpp:27-90). */
int pkt_runtime_initialize(pkt_runtime* rt, int max_tasks);
/* Copies the task list to the device and resets cursor, tokens and status (runtime.hpp:92-157). */
int pkt_runtime_submit(pkt_runtime* rt, const pkt_task* tasks, int n);
/* Stream-ordered variant: tasks from pinned host memory, no host sync. */
int pkt_runtime_submit_async(pkt_runtime* rt, const pkt_task* tasks, int n, void* stream);
/* Segments are accepted and kept as scheduling hints (runtime.hpp:159-173). */
int pkt_runtime_set_segments(pkt_runtime* rt, const int* begin_end_pairs, int n);
int pkt_runtime_set_segment_window_size(pkt_runtime* rt, int window);
/* One persistent launch over the submitted list (runtime.hpp:175-228). num_blocks <= 0: one CTA per SM. */
int pkt_runtime_launch(pkt_runtime* rt, int num_blocks, void* stream);
int pkt_runtime_synchronize(pkt_runtime* rt);
/* Device status word of the last launch: code (PKT_DEV_*), task index, token. */
int pkt_runtime_status(pkt_runtime* rt, int* code, int* task_index, int* detail);
/* Registers GEMM descriptors (builds their TMA tensor maps); returns the first id in *first_id. */
int pkt_runtime_register_gemms(pkt_runtime* rt, const pkt_gemm_desc* descs, int n, int* first_id);
int pkt_runtime_clear_gemms(pkt_runtime* rt);
/* Number of tiles of a registered GEMM (tiles_m * tiles_n). */
int pkt_gemm_tiles(const pkt_gemm_desc* d, int* tiles_m, int* tiles_n);
/* Wait budget of every device-side spin, in nanoseconds (default 2e9). */
int pkt_runtime_set_timeout_ns(pkt_runtime* rt, unsigned long long ns);
/* Launch mode: 1 = one CTA per SM works alone (default); 2 = CTA pairs (clusters of
 * two SMs) share 256-row GEMM tiles. pkt_runtime_launch clamps the grid to the CTAs
 * that can be resident at once and, in pair mode, rounds it to whole clusters. */
int pkt_runtime_set_cta_pair(pkt_runtime* rt, int pair);
int pkt_runtime_set_task_accounting(pkt_runtime* rt, int enabled);
int pkt_runtime_fetch_task_counter(pkt_runtime* rt, unsigned long long* out);
int pkt_runtime_set_perf(pkt_runtime* rt, int enabled);
/* Per-CTA role cycle counters of the last launch: blocks x PKT_PERF_WORDS u64. */
#define PKT_PERF_WORDS 16
int pkt_runtime_fetch_perf(pkt_runtime* rt, unsigned long long* out, int max_blocks, int* blocks);
int pkt_runtime_last_launch_blocks(pkt_runtime* rt);
/* For launching the megakernel instantiated with a program's own pk::OpTraits ops
 * (pk/kernel.cuh, pk::launch_with_ops; no counterpart in pkt, whose ops are
 * compiled into its one kernel): prepares the submitted list exactly as
 * pkt_runtime_launch does (grid clamped to the resident CTAs, counters cleared on
 * `stream`) and returns the kernel's parameter block (kparams_bytes must equal the
 * caller's sizeof(pkb::KParams)), the grid and the CTA-pair mode. */
int pkt_runtime_prepare_launch(pkt_runtime* rt, int num_blocks, void* stream, void* kparams, int kparams_bytes,
                               int* blocks, int* pair);
/* Effective SM clock of the launches since the last reset (no counterpart in pkt):
 * out3 = {SM cycles, nanoseconds, launches} summed over CTA 0's lifetime in every
 * launch; cycles * 1000 / ns is the mean SM clock in MHz. reset != 0 clears the
 * sums after reading them (out3 may be NULL to clear only). */
int pkt_runtime_clock_stats(pkt_runtime* rt, unsigned long long* out3, int reset);
/* Per-task trace of launches (no counterpart in pkt; its closest is the per-role
 * PerfBlock cycle counters): when enabled, every launch records for each task
 * PKT_TRACE_WORDS u64 = {CTA | opcode << 16 (GEMM tiles also: GEMM id << 32,
 * tile_m & 255 << 48, tile_n & 255 << 56), then %globaltimer ns at: dequeue, dependencies
 * satisfied, first TMA load issued, first MMA issued, last MMA committed, compute
 * warps started (GEMM: accumulator complete), compute warps finished}; stages a
 * task does not have stay 0. fetch copies the last launch's records (synchronous). */
#define PKT_TRACE_WORDS 8
int pkt_runtime_set_trace(pkt_runtime* rt, int enabled);
int pkt_runtime_fetch_trace(pkt_runtime* rt, unsigned long long* out, int max_tasks, int* n);
int pkt_num_sms(int device);
const char* pkt_last_error(void);

/* ---- axpy entry point (pkt examples/axpy_example.cu) --------------------- */
/* y = a*x + y over n floats on device memory, as one streaming task list. */
int pkt_axpy(const float* x, float* y, float a, long long n, void* stream);
/* Same result as pkt_axpy for callers that must not allocate device memory
 * (no counterpart in pkt: its runtime always cudaMallocs its task list). The
 * task list and status words live in a fixed ~192 KB array inside the library;
 * n is limited to 67,108,864 floats (larger n: PKT_ERR_ARGS, nothing launched).
 * Calls on one device share that array, so calls that overlap on the GPU race;
 * order them on one stream. The first call on a device looks up the array's
 * address and should come before any stream capture. */
int pkt_axpy_noalloc(const float* x, float* y, float a, long long n, void* stream);
/* Device status words of the last pkt_axpy_noalloc launch on the current device
 * (code PKT_DEV_*, task index, detail; all 0 when it ran cleanly), read from the
 * same fixed array without allocating. Synchronises the device first, so call it
 * after the work to check, not inside a stream capture. Every wait in that launch
 * has a fixed budget of 2 s; a launch that ran out of it reports
 * PKT_DEV_TIMEOUT_PIPE or PKT_DEV_TIMEOUT_DEPS here. The next pkt_axpy_noalloc
 * call clears the words. */
int pkt_axpy_noalloc_status(int* code, int* task_index, int* detail);

/* ---- MLP training engine (the hot path) -------------------------------- */
typedef struct pkt_mlp pkt_mlp;

typedef struct pkt_mlp_config {
  int num_layers;   /* L */
  const int* dims;  /* L+1 layer widths, dims[0] = input, dims[L] = output */
  int batch;        /* rows per GPU per step */
  int dtype;        /* PKT_DTYPE_BF16 (bf16 weights/acts, fp32 master) or PKT_DTYPE_TF32 */
  int has_bias;
  int relu_last;    /* ReLU after the output layer too (0 for plain regression) */
  float lr;
  int grad_mode;    /* 0: SGD fused into the weight-gradient epilogue; 1: store fp32
                       gradients, separate SGD pass (data parallel over NCCL /
                       inspection); 2: fused data parallel over peer memory
                       (pkt_mlp_dp_handle / pkt_mlp_dp_connect) */
  int max_bn;       /* largest tile N to use (0: 256) */
  int cta_pair;     /* 2: CTA pairs share 256-row tiles (tcgen05 cta_group::2);
                       1: every CTA computes its own 128-row tiles; 0: automatic
                       (pairs when the widest layer gives every pair a 256 x 256
                       tile, single CTAs for narrow, latency-bound networks) */
} pkt_mlp_config;

int pkt_mlp_create(int device, const pkt_mlp_config* cfg, pkt_mlp** out);
int pkt_mlp_destroy(pkt_mlp* m);
/* Parameters as fp32 host arrays: W concatenated [d_{l+1}, d_l] row-major, b concatenated. */
int pkt_mlp_set_params(pkt_mlp* m, const float* W, const float* b);
int pkt_mlp_get_params(pkt_mlp* m, float* W, float* b);
/* Gradients of the last step (grad_mode 1 only). */
int pkt_mlp_get_grads(pkt_mlp* m, float* dW, float* db);
/* Batch upload: x [batch, d0], target [batch, dL], host or device memory, in the
 * engine's storage type (uint16 bf16 bits for PKT_DTYPE_BF16, fp32 for TF32).
 * Stream-ordered (host memory should be pinned for async copies). The engine
 * has two input slots: each call fills the slot the previous call did not use
 * and makes it the one later training steps read, so a copy on another stream
 * can overlap the step still reading the other slot (the caller orders the
 * copy after the step that last read its slot, two loads back). */
int pkt_mlp_load_batch(pkt_mlp* m, const void* x, const void* target, int on_device, void* stream);
/* Enqueue `steps` training steps on the loaded batch. */
int pkt_mlp_train(pkt_mlp* m, int steps, void* stream);
/* Loss of each enqueued step since the last reset (device -> host, syncs). */
int pkt_mlp_losses(pkt_mlp* m, float* out, int max_n, int* n);
int pkt_mlp_reset_losses(pkt_mlp* m);
/* Device pointer of the loss of step i (for async reads). */
int pkt_mlp_loss_ptr(pkt_mlp* m, int i, float** out);
/* Output activations of the last step: y = last layer (fp32), [batch, dL]. */
int pkt_mlp_get_output(pkt_mlp* m, float* y);
int pkt_mlp_status(pkt_mlp* m, int* code, int* task_index, int* detail);
/* Tasks and GEMM tiles one step enqueues (for accounting). */
int pkt_mlp_step_info(pkt_mlp* m, int* tasks, int* gemm_tiles, double* flops);
/* Capture y = output layer (fp32) during training steps, for pkt_mlp_get_output. */
int pkt_mlp_set_output_capture(pkt_mlp* m, int enabled);
/* Data parallel (grad_mode 1). One step = pkt_mlp_forward_backward, then an
 * all-reduce (sum) of the fp32 gradient buffer by the caller (NCCL on the same
 * stream), then pkt_mlp_apply_update. grad_scale multiplies lr in the update
 * (1/world_size turns the summed per-rank mean gradients into the global mean). */
int pkt_mlp_grad_buffer(pkt_mlp* m, float** ptr, long long* count);
int pkt_mlp_set_grad_scale(pkt_mlp* m, float scale);
int pkt_mlp_forward_backward(pkt_mlp* m, void* stream);
int pkt_mlp_apply_update(pkt_mlp* m, void* stream);
/* The same step as pkt_mlp_forward_backward in L launches (grad_mode 1), so the
 * caller can all-reduce each layer's gradient on another stream as soon as it is
 * complete, overlapped with the rest of the backward: after segment s (0..L-1)
 * the bucket of layer L-1-s (pkt_mlp_grad_bucket: offset and count in floats
 * within pkt_mlp_grad_buffer, dW then db) is final. Segment 0 also runs the
 * forward and the loss. pkt_mlp_set_reserved_sms leaves that many SMs out of
 * the persistent grid, so a collective kernel on another stream has SMs to run
 * on while a segment runs (0 by default). */
int pkt_mlp_backward_segments(pkt_mlp* m, int* count);
int pkt_mlp_forward_backward_segment(pkt_mlp* m, int segment, void* stream);
int pkt_mlp_grad_bucket(pkt_mlp* m, int layer, long long* offset, long long* count);
int pkt_mlp_set_reserved_sms(pkt_mlp* m, int sms);
/* Fused data parallel (grad_mode 2): one launch per step on every rank; the
 * weight-gradient tiles go to their owner rank (tile index mod world) over
 * peer memory as they finish, the owner sums the ranks' partials in rank
 * order, applies SGD (lr x grad_scale) to its shard of the fp32 masters and
 * writes the new bf16 weights into every rank; the next step's forward tiles of
 * a layer start once that layer's weights have all arrived. Set-up: every rank
 * creates its engine, exports its exchange region (pkt_mlp_dp_handle, 64 bytes
 * of CUDA IPC handle), the caller exchanges the handles (e.g. an all-gather over
 * torch.distributed) and passes them, in rank order, to pkt_mlp_dp_connect.
 * world = 1 needs no handles. All ranks must run the same number of steps;
 * a rank that stops early makes the others' waits time out (PKT_ERR_TIMEOUT). */
#define PKT_DP_MAX_RANKS 8
int pkt_mlp_dp_handle(pkt_mlp* m, void* handle64);
int pkt_mlp_dp_connect(pkt_mlp* m, int rank, int world, const void* handles);
/* Per-CTA role cycle counters of the last launch (same layout as pkt_runtime_fetch_perf). */
int pkt_mlp_set_perf(pkt_mlp* m, int enabled);
int pkt_mlp_fetch_perf(pkt_mlp* m, unsigned long long* out, int max_blocks, int* blocks);
/* Effective SM clock of the engine's launches, as pkt_runtime_clock_stats. */
int pkt_mlp_clock_stats(pkt_mlp* m, unsigned long long* out3, int reset);
/* Per-task trace of the engine's launches, as pkt_runtime_set_trace / _fetch_trace
 * (task indices are those of one step's task list). */
int pkt_mlp_set_trace(pkt_mlp* m, int enabled);
int pkt_mlp_fetch_trace(pkt_mlp* m, unsigned long long* out, int max_tasks, int* n);

#ifdef __cplusplus
}
#endif

#endif /* PKT_B200_H */
