/*
 * ferro_cuda.h -- C ABI of the B200 (sm_100a) execution backend for
 * ferrograd's MLP training path.
 *
 * Every entry point returns an int status: 0 (FG_OK) on success, otherwise an
 * FG_ERR_* code, with a human-readable message available from
 * fg_last_error() on the calling thread.  No entry point aborts the process.
 * Pointers named d_* are device (HBM) pointers; h_* are host pointers.
 * Streams are cudaStream_t passed as void* (NULL = the legacy default stream).
 *
 * Each declaration cites the reference interface it replaces (file:line in
 * the ferrograd crate).
 */
#ifndef FERRO_CUDA_H
#define FERRO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum fg_status {
  FG_OK = 0,
  FG_ERR_INVALID = 1,    /* bad argument (size mismatch, null pointer, bad shape) */
  FG_ERR_CUDA = 2,       /* CUDA runtime / driver call failed */
  FG_ERR_COMPILE = 3,    /* NVRTC compilation failed (log in fg_last_error) */
  FG_ERR_NCCL = 4,       /* NCCL call failed or timed out */
  FG_ERR_DEVICE = 5,     /* a kernel reported an error word (bounded wait expired) */
  FG_ERR_UNSUPPORTED = 6 /* shape/layout this build does not handle */
};

/* dtype codes: src/dtype.rs:19-58 (F32, I32, Bool). */
enum fg_dtype { FG_F32 = 0, FG_I32 = 1, FG_BOOL = 2 };

/* reduce ops: ReduceAxis(Add) / ReduceAxis(Max), src/uop.rs:26-310. */
enum fg_reduce_op { FG_REDUCE_SUM = 0, FG_REDUCE_MAX = 1 };

typedef struct fg_device fg_device;
typedef struct fg_buffer fg_buffer;
typedef struct fg_program fg_program;
typedef struct fg_comm fg_comm;
typedef struct fg_mlp fg_mlp;

/* KernelArg (src/device.rs:241-251): tagged union {Buffer, I32, F32, Bool}. */
enum fg_arg_kind { FG_ARG_BUFFER = 0, FG_ARG_I32 = 1, FG_ARG_F32 = 2, FG_ARG_BOOL = 3 };
typedef struct fg_kernel_arg {
  int32_t kind;
  union {
    fg_buffer *buffer;
    int32_t i32;
    float f32;
    uint8_t b;
  } v;
} fg_kernel_arg;

/* Message of the last failing call on this thread ("" if none). */
const char *fg_last_error(void);

/* ---- Device trait (src/device.rs:275-332) ------------------------------ */

/* device::get(DeviceId::Cuda(ordinal)) (src/device.rs:338-354): opens the
 * device context and its stream.  One handle per ordinal per process. */
int fg_device_open(int ordinal, fg_device **out);
int fg_device_close(fg_device *dev);
/* Stream that buffer copies and fg_execute launches are ordered on. */
int fg_device_stream(fg_device *dev, void **stream);
int fg_device_sync(fg_device *dev);
/* Device-side timing (the CUDA counterpart of the per-kernel wall-clock
 * timing of DEBUG >= 2, src/tensor.rs:1017-1028): an event records a point
 * on a stream (NULL = the device's stream); fg_event_elapsed_ms waits for
 * `end` and returns the milliseconds between the two points. */
typedef struct fg_event fg_event;
int fg_event_create(fg_device *dev, fg_event **out);
int fg_event_record(fg_event *ev, void *stream);
int fg_event_elapsed_ms(fg_event *start, fg_event *end, float *ms);
int fg_event_destroy(fg_event *ev);

/* Device::allocate (src/device.rs:282-283): zero-initialised buffer of
 * numel elements of dtype.  numel == 0 is allowed (no storage). */
int fg_alloc(fg_device *dev, int dtype, size_t numel, fg_buffer **out);
/* Drop of the last Rc<BufferInner> (src/device.rs:95-105). */
int fg_free(fg_buffer *buf);
int fg_buffer_info(const fg_buffer *buf, void **d_ptr, int *dtype, size_t *numel);
/* Device::copy_from_host (src/device.rs:294, src/device/cpu.rs:283-302):
 * fails with "copy_from_host: expected N bytes, got M" on a size mismatch.
 * The copy is ordered on the device stream; h_src may be reused as soon as
 * the call returns. */
int fg_copy_h2d(fg_buffer *buf, const void *h_src, size_t nbytes);
/* Device::copy_to_host (src/device.rs:302, src/device/cpu.rs:304-316):
 * synchronous, like the reference's Vec<u8> return. */
int fg_copy_d2h(const fg_buffer *buf, void *h_dst, size_t nbytes);

/* Device::compile (src/device.rs:309-314): CUDA C source (extern "C"
 * __global__ func_name) compiled by NVRTC straight to an sm_100a cubin.
 * block/grid are the launch shape the renderer chose.  Compile errors return
 * FG_ERR_COMPILE with the NVRTC log in fg_last_error(). */
int fg_compile(fg_device *dev, const char *source, const char *func_name, int num_args,
               const uint32_t grid[3], const uint32_t block[3], fg_program **out);
int fg_program_free(fg_program *prog);
/* Device::execute (src/device.rs:321, src/device/cpu.rs:328-380): launches
 * on the device stream; fails if nargs != num_args. */
int fg_execute(fg_program *prog, const fg_kernel_arg *args, int nargs);

/* ---- Parameter init (src/nn.rs:12-47) ---------------------------------- */
/* kaiming_normal: the reference's LCG (s = s*6364136223846793005 + 1,
 * u = (s >> 33) / 2^31) feeding Box-Muller pairs (cos then sin) scaled by
 * sqrt(2 / fan_in), in f32 on the host.  *state carries the thread-local seed
 * across layers (42 at start, src/nn.rs:12-14); Linear::new (src/nn.rs:77-85)
 * draws its weight from it and zero-fills the bias. */
int fg_kaiming_normal(float *h_out, size_t numel, size_t fan_in, uint64_t *state);

/* ---- Fused building blocks the CUDA pattern router targets -------------- */
/* Elementwise relu(a*b+c)*scale over n f32 elements: the proto-kernels of
 * Tensor::mul/add/relu (src/tensor.rs:471-491,519-531) as one pass. */
int fg_ew_fma_relu_scale(const float *d_a, const float *d_b, const float *d_c, float *d_out,
                         size_t n, float scale, void *stream);

/* ReduceAxis over the last axis (Tensor::sum / Tensor::max,
 * src/tensor.rs:665-693): out[r] = op over x[r, 0..cols). */
int fg_reduce_rows(int dtype, int op, const void *d_x, void *d_out, size_t rows, size_t cols,
                   void *stream);
/* ReduceAxis over axis 0: out[c] = op over x[0..rows, c]; deterministic. */
int fg_reduce_cols(int dtype, int op, const void *d_x, void *d_out, size_t rows, size_t cols,
                   void *stream);

/* Tensor::cross_entropy (src/tensor.rs:738-752) forward and the gradient
 * autograd builds for it (src/gradient.rs:97-205), fused in one pass:
 * d_loss[0] = mean over rows of -sum_c t*log_softmax(x); d_dx (may be NULL)
 * = d loss / d x scaled by grad_scale (1.0 for the plain loss). */
int fg_xent_fwd_bwd(const float *d_logits, const float *d_targets, size_t rows, size_t cols,
                    float *d_loss, float *d_dx, float grad_scale, void *stream);

/* No counterpart in the reference.  fg_xent_fwd_bwd without any device
 * allocation, for callers that may not allocate device memory after start-up
 * (a process that reserves its whole memory budget up front: cudaMalloc can
 * synchronise the device and fail under fragmentation mid-run).  The per-row
 * scratch is a static array inside the library, 1 MiB on every GPU that
 * loads it, so rows is limited to FG_XENT_NOALLOC_MAX_ROWS; larger inputs
 * return FG_ERR_INVALID.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) and should come before any stream
 * capture.  Under lazy module loading (the CUDA default since 12.2) that
 * first call, or the first launch of any kernel of this library on the
 * device, also loads the library's device code, which allocates the array
 * and the code itself: make one warm-up call per device at start-up, before
 * reserving the memory budget (or run with CUDA_MODULE_LOADING=EAGER).
 * Later calls allocate nothing.  All calls share the array: calls that
 * overlap on the GPU race. */
#define FG_XENT_NOALLOC_MAX_ROWS 262144
int fg_xent_fwd_bwd_noalloc(const float *d_logits, const float *d_targets, size_t rows,
                            size_t cols, float *d_loss, float *d_dx, float grad_scale,
                            void *stream);

/* Sgd::step (src/optim.rs:60-71): p <- p + (-(g*lr)).  If d_p_lo is not
 * NULL it also receives the TF32 residual of the updated p (see fg_split_lo). */
int fg_sgd(float *d_p, const float *d_g, size_t n, float lr, float *d_p_lo, void *stream);

/* Dataset path.  parse_images (src/dataset.rs:116-140) maps each IDX pixel
 * to f32::from(b) / 255.0; here the bytes are uploaded once and converted on
 * the device: d_dst[i] = (float)d_src[i] / divisor, correctly rounded (the
 * same value).  one_hot (examples/mnist.rs:7-14): d_out[i, c] = 1.0 when
 * d_labels[i] == c, else 0.0 ([n, classes], row-major); a label >= classes
 * leaves its row all zero (the host loader rejects such labels first). */
int fg_u8_to_f32_div(const uint8_t *d_src, float *d_dst, size_t n, float divisor, void *stream);
int fg_one_hot_u8(const uint8_t *d_labels, float *d_out, size_t n, int classes, void *stream);

/* TF32 residual: lo[i] = x[i] - (x[i] with its low 13 mantissa bits cleared).
 * The tensor cores read x itself as the high part. */
int fg_split_lo(const float *d_x, float *d_lo, size_t n, void *stream);

/* GEMM epilogues. */
enum fg_gemm_epilogue {
  FG_EPI_NONE = 0,      /* C = acc */
  FG_EPI_BIAS = 1,      /* C = acc + bias[n] */
  FG_EPI_BIAS_RELU = 2, /* C = relu(acc + bias[n]) */
  FG_EPI_RELU_MASK = 3  /* C = (mask[m,n] > 0) ? acc : 0 */
};
/* Operand layout flags. */
enum fg_gemm_flags {
  FG_GEMM_A_MN_MAJOR = 1, /* A stored [K, M] (M contiguous) instead of [M, K] */
  FG_GEMM_B_MN_MAJOR = 2, /* B stored [K, N] (N contiguous) instead of [N, K] */
  FG_GEMM_1XTF32 = 4      /* drop the residual products (plain TF32) */
};
/* The reduce-of-broadcast-mul behind Tensor::matmul (src/tensor.rs:762-778)
 * and its two backward contractions (src/gradient.rs:100-106,165-176):
 *   C[m,n] = sum_k A(m,k) * B(n,k)
 * on the tcgen05 tensor cores in 3xTF32 (hi*hi + hi*lo + lo*hi), fp32
 * accumulation in TMEM.  d_a_lo / d_b_lo are the TF32 residuals of A and B
 * in the same layout (fg_split_lo).  lda/ldb/ldc are row pitches in elements.
 * d_c_lo (may be NULL) receives the residual of C for a following GEMM.
 * Requirements: M, N, K > 0, pitches multiples of 4 elements, 16-byte
 * aligned pointers. */
int fg_gemm_3xtf32(int M, int N, int K, const float *d_a, const float *d_a_lo, int lda,
                   const float *d_b, const float *d_b_lo, int ldb, float *d_c, float *d_c_lo,
                   int ldc, int flags, int epilogue, const float *d_bias, const float *d_mask,
                   int ldmask, void *stream);

/* ---- MLP training step: forward -> cross_entropy -> backward -> Sgd ----- */
/* examples/mnist.rs:90-97 on the GPU.  Layers are Linear (src/nn.rs:67-104)
 * with ReLU between them; dims[0..n_layers] are the widths.  batch is the
 * rows this rank processes; with a communicator attached the gradients are
 * averaged across ranks before the update (data parallel). */
int fg_mlp_create(fg_device *dev, int n_layers, const int *dims, int batch, float lr,
                  fg_mlp **out);
int fg_mlp_destroy(fg_mlp *mlp);
/* Host <-> device parameter transfer; layer l weight is [dims[l+1], dims[l]]. */
int fg_mlp_set_params(fg_mlp *mlp, int layer, const float *h_weight, const float *h_bias);
int fg_mlp_get_params(fg_mlp *mlp, int layer, float *h_weight, float *h_bias);
int fg_mlp_get_grads(fg_mlp *mlp, int layer, float *h_dweight, float *h_dbias);
int fg_mlp_attach_comm(fg_mlp *mlp, fg_comm *comm);
/* Device pointers of the step's input slots ([batch, dims[0]] and
 * [batch, dims[n_layers]]) for callers that fill them on the GPU. */
int fg_mlp_input_slots(fg_mlp *mlp, float **d_x, float **d_targets);
/* One step on inputs already in the input slots; d_loss_out (device, may be
 * NULL) receives this step's loss (mean over the global batch). */
int fg_mlp_step(fg_mlp *mlp, float *d_loss_out);
/* One step from host memory: copies h_x / h_targets in, runs the step and
 * copies the loss out (blocking), the ferrograd call sequence
 * forward/backward/step/loss.to_vec(). */
int fg_mlp_step_host(fg_mlp *mlp, const float *h_x, const float *h_targets, float *h_loss);
/* fg_mlp_step_host with the next batch's upload overlapped: runs the step
 * on (h_x, h_targets) and returns its loss like fg_mlp_step_host, and while
 * the step computes, the copy engine uploads (h_x_next, h_targets_next) into
 * a second device staging slot.  A call whose (h_x, h_targets) are the
 * pointers the previous call named as its next batch uses that upload
 * instead of copying again; any other pair is uploaded first.  The training
 * loop of examples/mnist.rs:87-97 passes batch i+1 with batch i.  The next
 * batch's host buffers must stay unchanged until the following call
 * returns, and must be pinned (page-locked) for the copy to overlap.  Both
 * next pointers NULL: no prefetch. */
int fg_mlp_step_host_next(fg_mlp *mlp, const float *h_x, const float *h_targets,
                          const float *h_x_next, const float *h_targets_next, float *h_loss);
/* Capture the device part of fg_mlp_step in a CUDA graph and replay it. */
int fg_mlp_use_graph(fg_mlp *mlp, int enable);
/* Pre-update logits of the last step, [batch, dims[n_layers]] (loss.to_vec()
 * reads pre-update values in the reference, src/tensor.rs:222-252). */
int fg_mlp_get_logits(fg_mlp *mlp, float *h_logits);
/* Output of layer `layer` in the last step's forward pass, [batch,
 * dims[layer+1]]: post-ReLU activations for hidden layers, logits for the
 * last (the intermediates ferrograd materializes, src/schedule.rs:289-335). */
int fg_mlp_get_activations(fg_mlp *mlp, int layer, float *h_out);
/* Launches of this library's kernels issued by the last fg_mlp_step. */
int fg_mlp_launch_count(fg_mlp *mlp, int *count);
/* GEMM timing: when enabled, each step records a CUDA event pair around every
 * tensor-core GEMM launch on the step's stream (kept inside the CUDA graph
 * when graph replay is on).  fg_mlp_gemm_times returns, for the most recent
 * step, each GEMM's duration in ms and its algorithmic flops (2*M*N*K);
 * capacity is the length of both arrays, *count the number written. */
int fg_mlp_enable_gemm_timing(fg_mlp *mlp, int enable);
int fg_mlp_gemm_times(fg_mlp *mlp, float *ms, double *flops, int capacity, int *count);
/* With GEMM timing enabled and a communicator attached: duration (ms, from
 * enqueue on the comm stream to completion) and size of each gradient
 * all-reduce of the most recent step. */
int fg_mlp_comm_times(fg_mlp *mlp, float *ms, double *bytes, int capacity, int *count);

/* ---- Peer-sharded data parallelism (no reference counterpart: the
 * reference is single-device, src/device.rs:37-41) -------------------------
 * The alternative to fg_mlp_attach_comm for ranks on GPUs of one NVLink
 * domain.  Gradients are cut into chunks (layer 0's dW into `chunks` row
 * blocks, every other layer one chunk); each chunk is split into nranks
 * shards and shard r belongs to rank r.  As soon as a chunk is complete a
 * rank copies every other rank's shard into that rank's staging area with
 * the copy engines (no SMs), the owner sums the nranks contributions in rank
 * order and applies the SGD update to its shard of the parameters in one
 * kernel, and copies the updated shard (and its TF32 residual) to every
 * peer.  Parameters are double-buffered (even steps read buffer 0 and write
 * buffer 1), so no rank overwrites weights a peer is still reading; ranks
 * order the phases through flag words in each other's memory, and every
 * wait is bounded (FG_ERR_DEVICE from fg_check_device_error on expiry).
 *
 * fg_mlp_peer_prepare: allocates this rank's exchange region (gradients,
 * staging, both parameter buffers, flags), moves the current parameters
 * into it and writes this rank's handle (FG_PEER_HANDLE_BYTES) to
 * handle_out.  fg_mlp_peer_connect: takes the nranks handles in rank order
 * and maps the peers' regions; from then on fg_mlp_step runs the sharded
 * schedule.  Every rank must call both (same dims, batch, nranks, chunks)
 * and run the same number of steps.  fg_mlp_get_grads then reads each rank's
 * reduced shard and must not overlap another rank's next step.  To shut
 * down, every rank calls fg_mlp_peer_disconnect (unmaps the peers' regions),
 * then all pass a host barrier, then each calls fg_mlp_destroy: a region
 * must not be freed while another rank still maps it.  Not combinable with
 * fg_mlp_attach_comm. */
#define FG_PEER_HANDLE_BYTES 96
int fg_mlp_peer_prepare(fg_mlp *mlp, int rank, int nranks, int chunks,
                        char handle_out[FG_PEER_HANDLE_BYTES]);
int fg_mlp_peer_connect(fg_mlp *mlp, const char *handles);
int fg_mlp_peer_disconnect(fg_mlp *mlp);
/* Host-only layout query for the sharded exchange (no GPU needed): floats in
 * a rank's exchange region, and the chunks' offsets and lengths (floats from
 * the start of the gradient area; at most `capacity` written, *n_chunks set
 * to the total). */
int fg_peer_layout(int n_layers, const int *dims, int nranks, int chunks, size_t *region_floats,
                   size_t *chunk_off, size_t *chunk_len, int capacity, int *n_chunks);
/* Host-only, same layout: where each layer's dW (w_off[l]) and db (b_off[l])
 * start in the gradient area (floats; n_layers entries each), and the loss
 * slot (*loss_off, inside layer 0's bucket, averaged with it). */
int fg_peer_layout_offsets(int n_layers, const int *dims, int nranks, int chunks, size_t *w_off,
                           size_t *b_off, size_t *loss_off);
/* The owner's pass of the sharded exchange for one chunk, run on this GPU
 * alone with every rank's contribution already in place (a test of the
 * exchange's kernels without a second GPU).  d_grad, d_stage, d_p_cur,
 * d_p_next and d_lo_next point at the chunk's start (nranks * shard floats
 * each): this rank's contribution is d_grad[rank*shard ..), sender j's is
 * d_stage[j*shard ..).  A one-block kernel waits until d_flags[j] == val for
 * every j != rank (d_flags: kMaxPeers = 8 words), at most wait_ms
 * milliseconds; then the owned shard of d_grad receives the sum of the
 * nranks contributions in rank order, d_p_next = d_p_cur + (-(g*lr))
 * (src/optim.rs:60-71) and d_lo_next its TF32 residual, except that the
 * element at loss_idx (chunk-relative, or -1) takes the summed value.  If
 * the wait gives up, nothing is written and the call returns FG_ERR_DEVICE
 * (the device error word).  Synchronous. */
int fg_peer_reduce_sgd_local(float *d_grad, const float *d_stage, const float *d_p_cur,
                             float *d_p_next, float *d_lo_next, size_t shard, int rank, int nranks,
                             float lr, long long loss_idx, const unsigned int *d_flags,
                             unsigned int val, int wait_ms, void *stream);

/* ---- Data-parallel communicator (no reference counterpart: the reference
 * is single-device, src/device.rs:37-41) ----------------------------------- */
#define FG_UNIQUE_ID_BYTES 128
int fg_comm_unique_id(char out[FG_UNIQUE_ID_BYTES]);
/* Non-blocking NCCL init polled until timeout_ms; on timeout the
 * communicator is aborted and FG_ERR_NCCL returned. */
int fg_comm_init(int rank, int nranks, const char uid[FG_UNIQUE_ID_BYTES], int timeout_ms,
                 fg_comm **out);
int fg_comm_destroy(fg_comm *comm);
int fg_comm_abort(fg_comm *comm);
/* In-place mean over ranks of count f32 values on stream. */
int fg_allreduce_mean_f32(fg_comm *comm, float *d_buf, size_t count, void *stream);

/* ---- Diagnostics -------------------------------------------------------- */
/* Reads and clears the device error word kernels set when a bounded wait
 * expires; returns FG_ERR_DEVICE with a description if it was set. */
int fg_check_device_error(void);
/* Total launches of this library's kernels in this process. */
uint64_t fg_kernel_launches(void);
/* Architecture the current device runs this library's kernels as:
 * cudaFuncGetAttributes' binaryVersion (100 for sm_100a) and ptxVersion (0
 * when no PTX is embedded).  Needs a GPU. */
int fg_kernel_arch(int *binary_version, int *ptx_version);

#ifdef __cplusplus
}
#endif
#endif /* FERRO_CUDA_H */
