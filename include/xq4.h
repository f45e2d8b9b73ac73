/*
 * xq4.h -- C ABI of the B200 (sm_100a) backend for xnpu's int4 ("w4" / Q4NX)
 * weight-matrix path.
 *
 * The reference (nzinfo/xnpu) drives this path through its HAL crate
 * (crates/xnpu-hal): open a device, create buffer objects, upload weights and
 * activations, submit one op packet whose arguments are [W, x, C], and wait on
 * a timeline point with a deadline.  Each entry point below replaces one piece
 * of that surface and names the reference item it stands in for.  All calls
 * return an int status (XQ4_OK on success); the message of the last failure
 * on the calling thread is available from xq4_last_error_string().
 *
 * Ownership: every handle is created by one call and released by exactly one
 * destroy/close call (the reference's RAII: Device owns fd + heap,
 * crates/xnpu-hal/src/accel.rs:107-116; BufferObject closes its handle on drop,
 * crates/xnpu-hal/src/bo.rs:160-181).  A weight or buffer may be destroyed
 * after its device was closed, but no op may use it after that.  Handles are
 * not thread-safe; use one
 * device handle (one in-order queue) per thread, as the reference does
 * (one in-order queue per context, crates/xnpu-cli/src/main.rs:1637-1641).
 *
 * Numerics: int4 codes q in [-8, 7] with one bf16 scale per 32 consecutive K
 * values of a row; dequantized weight w = RNE_bf16(f32(q) * f32(scale))
 * (crates/xnpu-cli/src/main.rs:3097-3125); y = sum_k w*x accumulated in f32,
 * rounded once to the output type (crates/xnpu-cli/src/main.rs:2287-2296).
 */
#ifndef XQ4_H
#define XQ4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
/* The reference reports std::io::Result errno (crates/xnpu-hal/src/ioctl.rs:59-66)
 * and a timeline-wait timeout as an error (crates/xnpu-hal/src/ert.rs:214-261). */
#define XQ4_OK 0
#define XQ4_EINVAL 1     /* bad argument, size, layout or alignment */
#define XQ4_ENOMEM 2     /* device or host allocation failed */
#define XQ4_ECUDA 3      /* CUDA runtime/driver error (message has the detail) */
#define XQ4_ETIMEDOUT 4  /* xq4_wait deadline passed before completion */
#define XQ4_ENCCL 5      /* NCCL error in the sharded path */
#define XQ4_ENOTSUP 6    /* valid request this build does not implement */
#define XQ4_ENODEV 7     /* no usable sm_100 device at that ordinal */

/* ---------------------------------------------------------------- layouts */
/* Source layouts accepted by xq4_weight_import. */
#define XQ4_LAYOUT_L1 1     /* w4gemv2 tile layout written by tools/w4_import.py
                               (crates/xnpu-cli/src/main.rs:2186-2252) */
#define XQ4_LAYOUT_L2 2     /* w4gemvu v4/v5 16x2048 block layout, the "Q4NX" pack
                               (crates/xnpu-cli/src/main.rs:2912-2949, :3097-3125) */
#define XQ4_LAYOUT_PLANES 3 /* row-major planes: codes [n][k/2] bytes (low nibble =
                               even k) then scales [n][k/group] at scale_offset */

#define XQ4_CODE_S4 0       /* nibble = two's-complement q (the reference's ABI) */
#define XQ4_CODE_U4_ZP8 1   /* nibble = q + 8, code in [0, 15], zero point 8 */

#define XQ4_SCALE_BF16 0
#define XQ4_SCALE_FP16 1    /* must be exactly representable in bf16 */

#define XQ4_OUT_BF16 0      /* output rounded RNE to bf16 */
#define XQ4_OUT_F32 1       /* output kept in f32 (logits) */

typedef struct xq4_layout_desc {
    int layout;        /* XQ4_LAYOUT_* */
    int n;             /* rows (output features) of the FULL matrix in src */
    int k;             /* reduction length; multiple of 32 */
    int group;         /* must be 32 */
    int tsi;           /* L1 only: rows per tile (16 or 4 in the reference) */
    int cols;          /* L1 only: column count (8 in the reference) */
    int code_format;   /* PLANES only: XQ4_CODE_* */
    int scale_dtype;   /* PLANES only: XQ4_SCALE_* */
    size_t scale_offset; /* PLANES only: byte offset of the scale plane in src */
    int row_begin;     /* import rows [row_begin, row_end) of src; both 0 = all */
    int row_end;
} xq4_layout_desc;

typedef struct xq4_device xq4_device;
typedef struct xq4_buffer xq4_buffer;
typedef struct xq4_weight xq4_weight;
typedef struct xq4_comm xq4_comm;

typedef struct xq4_device_info {
    int ordinal;
    int sm_count;
    int cc_major, cc_minor;
    size_t hbm_bytes;
    size_t l2_bytes;
    char name[96];
} xq4_device_info;

/* ---------------------------------------------------------------- errors */
/* Message of the last failing call on this thread ("" if none). */
const char *xq4_last_error_string(void);
/* Library version string. */
const char *xq4_version(void);

/* ---------------------------------------------------------------- device */
/* Replaces Device::open_default / Device::open (crates/xnpu-hal/src/accel.rs:122,
 * :144) plus HwContext::create + configure_cus (crates/xnpu-hal/src/hwctx.rs:28,
 * :95): binds CUDA device `ordinal`, creates its in-order stream and timeline. */
int xq4_device_open(int ordinal, xq4_device **out);
/* Replaces Device / HwContext drop (accel.rs:107-116, hwctx.rs:154-193). */
int xq4_device_close(xq4_device *dev);
/* Replaces Device::aie_metadata (crates/xnpu-hal/src/accel.rs:248). */
int xq4_device_query(const xq4_device *dev, xq4_device_info *info);
/* The device's in-order stream (a cudaStream_t), for callers that interleave
 * their own work; the reference's queue is per context (hwctx.rs:12). */
void *xq4_device_stream(xq4_device *dev);

/* ---------------------------------------------------------------- buffers */
/* Replaces BufferObject::new(dev, BoType, size) (crates/xnpu-hal/src/bo.rs:42).
 * Device memory, 256-byte aligned. */
int xq4_buffer_create(xq4_device *dev, size_t bytes, xq4_buffer **out);
/* Replaces write through Mapping + sync(ToDevice, off, len)
 * (crates/xnpu-hal/src/bo.rs:134, accel.rs:186).  Stream-ordered on the
 * device's queue; returns after the host copy is consumed. */
int xq4_buffer_upload(xq4_buffer *buf, const void *host, size_t offset, size_t len);
/* Replaces sync(FromDevice) + read through Mapping (bo.rs:134, accel.rs:209).
 * Waits for all queued work on the device first (in-order queue). */
int xq4_buffer_download(xq4_buffer *buf, void *host, size_t offset, size_t len);
/* Replaces BufferObject drop (crates/xnpu-hal/src/bo.rs:160-181). */
int xq4_buffer_destroy(xq4_buffer *buf);
/* Device address of the buffer; replaces BufferObject::xdna_addr (bo.rs:130). */
void *xq4_buffer_device_ptr(const xq4_buffer *buf);
size_t xq4_buffer_size(const xq4_buffer *buf);

/* ---------------------------------------------------------------- weights */
/* Offline import: repack src (host bytes, in `desc->layout`) into the GPU
 * layout and upload it.  Replaces the weight-buffer upload of the reference
 * (chain_tensor, crates/xnpu-cli/src/main.rs:1589-1603, over files written by
 * tools/w4_import.py:116-120) and its size check (main.rs:2597).  The
 * dequantized values are bit-identical to the source layout's.  The row range
 * selects a column shard of the matrix (the reference splits rows across its
 * 8 AIE columns, main.rs:2186-2191). */
int xq4_weight_import(xq4_device *dev, const void *src, size_t src_len,
                      const xq4_layout_desc *desc, xq4_weight **out);
int xq4_weight_destroy(xq4_weight *w);
/* Rows, reduction length and bytes resident in HBM for the weight. */
int xq4_weight_shape(const xq4_weight *w, int *n, int *k, size_t *device_bytes);
/* Repack only (no device): size of the GPU-layout image for n x k. */
size_t xq4_gpu_layout_bytes(int n, int k);
/* Repack only (no device): write the GPU-layout image of src rows
 * [row_begin,row_end) into dst (xq4_gpu_layout_bytes bytes). */
int xq4_repack_host(const void *src, size_t src_len, const xq4_layout_desc *desc,
                    void *dst, size_t dst_len);

/* Dequantize the whole weight to bf16, row-major [n][k], into device memory
 * at out_dev (n*k*2 bytes), on `stream` (a cudaStream_t; NULL = CUDA's
 * default stream, as in the CUDA API).
 * Restates w4u_row_bf16 (crates/xnpu-cli/src/main.rs:3102-3125) for every row. */
int xq4_dequant(const xq4_weight *w, void *out_dev, void *stream);

/* ---------------------------------------------------------------- the op */
/* y[m][n] = x[m][k] . dequant(W)^T.  Replaces building and submitting one
 * w4 GEMV op packet with args [W, x, C] (StartNpuCmd::new/arg64/submit,
 * crates/xnpu-hal/src/ert.rs:77-212; chain_op, crates/xnpu-cli/src/main.rs:
 * 1611-1635) and returns its timeline point in *seq (may be NULL).
 * x: bf16 [m][k] at x_off bytes into x_buf; y: [m][n] of out_dtype at y_off.
 * m <= 24 runs the decode GEMV kernel (16 tokens per launch), m >= 25 the
 * tensor-core GEMM. */
int xq4_linear(xq4_device *dev, const xq4_weight *w,
               const xq4_buffer *x_buf, size_t x_off,
               xq4_buffer *y_buf, size_t y_off,
               int m, int out_dtype, uint64_t *seq);

/* Same op on raw device pointers and a caller stream (a cudaStream_t; NULL =
 * CUDA's default stream, as in the CUDA API; the device queue of xq4_linear
 * is xq4_device_stream()).  x and y must be 16-byte aligned. */
int xq4_linear_raw(const xq4_weight *w, const void *x_dev, void *y_dev,
                   int m, int out_dtype, void *stream);

/* ---------------------------------------------------------------- op chains */
/* A prebuilt chain of GEMV ops run as ONE persistent kernel: the weights of
 * the next op stream in while the current op finishes, so a decode step's
 * projections pay one launch ramp and tail instead of one per op.  Replaces
 * the reference's chained op packets built once and submitted together
 * (chain_op, crates/xnpu-cli/src/main.rs:1611-1635; the projection stream of
 * cmd_run_w4layer, main.rs:2487-2499).  Ops run in order; an op with
 * wait_prev != 0 reads its x only after the previous op's y is completely
 * written (so x may be an earlier op's output); wait_prev = 0 lets the op
 * start while the previous one is still finishing (independent inputs).
 * Each op: m in 1..8, out_dtype XQ4_OUT_BF16/F32, x 16-byte aligned, y
 * aligned to its element.  The op table is copied to the device at create;
 * the pointers must stay valid while the chain is used.  A chain runs on one
 * stream at a time (its completion counters are per chain).  A dependency
 * wait that runs out (2 s) sets fault bit 0x10.  The kernel's CTAs (2 per SM)
 * wait for one another, so all of them must be resident at once: create
 * returns XQ4_ENOTSUP when the device cannot hold them (the environment
 * variable XQ4_RESIDENT_CTAS_PER_SM, for diagnostics, replaces the occupancy
 * figure this check uses).  With a sharded op, run and submit return
 * XQ4_ETIMEDOUT once the communicator is unusable (see
 * xq4_linear_sharded_fused). */
typedef struct xq4_chain xq4_chain;
typedef struct xq4_chain_op {
    const xq4_weight *w;
    const void *x_dev;
    void *y_dev;
    int m;
    int out_dtype;
    int wait_prev;
    /* NULL, or the communicator over which the op is column-sharded as
     * xq4_linear_sharded_fused: w is this rank's row shard (every rank's of
     * the same size), y_dev the full m x n_total output (m x n_total/2 with
     * swiglu: each rank computes the SwiGLU of its own row pairs and the
     * intermediate is what is gathered).  A rank's rows reach the peers'
     * inboxes while the chain runs; each rank copies the peers' rows into
     * y_dev before the next op that waits, or at the end of the launch.  All
     * sharded ops of a chain use one communicator, their m x n_total
     * (n_total/2 with swiglu) summed is at most XQ4_FUSED_MAX_VALUES, and
     * every rank creates and runs its chain (the same op shapes, on GPUs
     * with the same SM count) together with the others: create is
     * collective when it maps the inboxes, as the first
     * xq4_linear_sharded_fused call.  A sharded op takes no residual. */
    struct xq4_comm *comm;
    /* Decode-step glue fused into the op (NULL / 0 = none; not with comm),
     * each as the reference computes it (crates/xnpu-cli/src/main.rs:
     * 4714-4745):
     *   norm_w_dev: x is RMS-normalised per token with these k bf16 weights
     *     before the product, RNE_bf16(x * inv * w) with inv = 1 /
     *     sqrt(mean(x^2) + norm_eps) (rms_norm_bf16); x must be an
     *     activation no op of the chain writes;
     *   residual_dev: y = RNE_bf16(RNE_bf16(W x) + residual), residual bf16
     *     [m][n] (add_bf16; it may be an earlier op's y when a wait_prev lies
     *     between them); bf16 output only;
     *   swiglu: the weight's rows alternate gate_i, up_i (an interleaved
     *     gate/up projection, n even); y is bf16 [m][n/2] with
     *     y[i] = RNE_bf16(g * (1 / (1 + exp(-g))) * u) of the op's bf16
     *     outputs g = row 2i, u = row 2i+1 (swiglu_bf16). */
    const void *norm_w_dev;
    float norm_eps;
    const void *residual_dev;
    int swiglu;
    /* Non-zero: the op runs in the W4A8 parity mode of xq4_linear_w4a8 (the
     * reference's NPU numerics): the chain's prep quantizes x -- after the
     * RMSNorm, when norm_w_dev is given: the reference's fused rms -> quant
     * -> GEMV pair, crates/xnpu-cli/src/main.rs:7802-7815 -- per 32-K group
     * to int8 exactly as xq4_quantize_x (w4u_quantize_x, main.rs:2955-2986),
     * and the op's output is the xq4_linear_w4a8 result for it, bit for bit.
     * x must be an activation no op of the chain writes. */
    int w4a8;
} xq4_chain_op;
int xq4_chain_create(xq4_device *dev, const xq4_chain_op *ops, int n_ops, xq4_chain **out);
int xq4_chain_destroy(xq4_chain *chain);
/* Submit on the device queue (after everything queued before); timeline
 * point in *seq (may be NULL), as xq4_linear. */
int xq4_chain_submit(xq4_device *dev, const xq4_chain *chain, uint64_t *seq);
/* Run on a caller stream (a cudaStream_t; NULL = CUDA's default stream). */
int xq4_chain_run(const xq4_chain *chain, void *stream);

/* Replaces syncobj_timeline_wait(dev, syncobj, seq, timeout_ns)
 * (crates/xnpu-hal/src/ert.rs:218) and the completed-state check
 * (ert.rs:147-151): XQ4_OK when the op at `seq` and everything queued before
 * it has completed, XQ4_ETIMEDOUT if timeout_ns elapsed first (the work stays
 * queued and a later wait may succeed), XQ4_ECUDA if the device reported an
 * error.  The calling thread polls without sleeping for the first 2 ms, then
 * sleeps 20 us between polls. */
int xq4_wait(xq4_device *dev, uint64_t seq, int64_t timeout_ns);
/* Timeline point of the newest submitted op. */
uint64_t xq4_last_seq(const xq4_device *dev);
/* Read and clear the device's pipeline-fault bits.  Every wait inside the
 * kernels is bounded; a kernel whose wait runs out (a pipeline that stopped
 * making progress) sets a bit here and returns instead of hanging the GPU.
 * The reference's counterpart is the firmware health-data / ERT state check
 * (crates/xnpu-hal/src/ert.rs:147-165).  *bits = 0 means no fault. */
int xq4_device_fault(xq4_device *dev, uint32_t *bits);

/* ---------------------------------------------------------------- W4A8 parity mode */
/* The reference's NPU numerics (its w4gemvu kernel takes int8 activations).
 * Quantize bf16 x [m][k] (device) to int8 q [m][k] and bf16 group scales
 * d [m][k/32]: per 32-K group d = RNE_bf16(max|x| / 127),
 * q = clamp(round_half_even(x / d), -127, 127); an all-zero group gives q = 0,
 * d = 0.  Bit-exact with w4u_quantize_x (crates/xnpu-cli/src/main.rs:
 * 2955-2986).  Runs on CUDA device `device`, on `stream` (NULL = default). */
int xq4_quantize_x(const void *x_dev, int m, int k, void *q_dev, void *d_dev, int device, void *stream);
/* y[m][n] from the int8 activations of xq4_quantize_x: per 32-K group the
 * exact int32 dot of q_x with the int4 weights, times f32(s_w) * f32(d_x),
 * accumulated in f32 over each 2048-K chunk; each chunk partial is rounded
 * to bf16 (the NPU writes its C tensor as bf16, main.rs:2912-2916) and the
 * partials are summed in f32 in chunk order (w4u_read_c, main.rs:3066-3091),
 * then rounded to out_dtype.  q must be 16-byte aligned. */
int xq4_linear_w4a8(const xq4_weight *w, const void *q_dev, const void *d_dev, void *y_dev, int m,
                    int out_dtype, void *stream);

/* ---------------------------------------------------------------- decode attention */
/* The attention side of a decode step, one launch per layer, standing in for
 * the reference's host glue of its decode loop: rope_table + rope_apply
 * (crates/xnpu-cli/src/main.rs:4817-4839), the per-head q/k RMSNorm
 * qk_rms_bf16 (main.rs:4844-4857) and the GQA decode attention
 * attention_bf16 (main.rs:4967-5033).  Head dim 128.  An xq4_attn holds the
 * RoPE table (every position of the cache, computed on the host with the
 * reference's f32 formula: base^(-j/64), cos/sin of pos * that), the split
 * partials and the merge counters of one attention shape; calls on one
 * xq4_attn must not overlap on the GPU (one stream). */
typedef struct xq4_attn xq4_attn;
/* heads q heads over nkv kv heads (heads % nkv == 0, at most 8 q heads per kv
 * head), caches of cache_seq positions; rope_base 0 = no RoPE. */
int xq4_attn_create(xq4_device *dev, int heads, int nkv, int cache_seq, float rope_base, xq4_attn **out);
int xq4_attn_destroy(xq4_attn *attn);
/* For the token at position *pos_dev (device int, 0 <= pos < cache_seq; read
 * by the kernel, so a CUDA graph can replay the call as pos advances):
 * qkv_dev bf16 [heads*128 | nkv*128 k | nkv*128 v] is the token's qkv
 * projection output.  q and k are rotated by RoPE (one bf16 rounding) and,
 * when q_norm_w_dev / k_norm_w_dev (bf16 [128], shared by the heads; NULL =
 * none) are given, RMS-normalised per head; k and v are written into the
 * caches (bf16 [nkv][cache_seq][128]) at pos; out_dev (bf16 [heads*128])
 * receives, per q head h, softmax((K q_h) / sqrt(128)) . V over positions
 * 0..pos of kv head h / (heads / nkv), in f32, rounded once.  qkv and the
 * caches 16-byte aligned, out 8-byte aligned.  A position outside the cache
 * writes nothing and sets fault bit 0x20 (xq4_device_fault).  Runs on
 * `stream` (cudaStream_t; NULL = CUDA's default stream). */
int xq4_attn_decode(xq4_attn *attn, const void *qkv_dev, const void *q_norm_w_dev, const void *k_norm_w_dev,
                    void *k_cache_dev, void *v_cache_dev, const int *pos_dev, void *out_dev, void *stream);

/* ---------------------------------------------------------------- shards */
/* Column (N) sharding of large-N projections over P GPUs with an NCCL
 * all-gather of the outputs.  The reference is single-device; its nearest
 * counterpart is the row split over AIE columns with a host gather of the
 * per-column C sections (w4u_read_c, crates/xnpu-cli/src/main.rs:3066-3091). */
#define XQ4_UNIQUE_ID_BYTES 128
int xq4_comm_unique_id(void *id_out /* XQ4_UNIQUE_ID_BYTES */);
int xq4_comm_init(xq4_device *dev, int rank, int nranks, const void *unique_id,
                  xq4_comm **out);
int xq4_comm_destroy(xq4_comm *comm);
/* y_full[m][n_total] = x . W^T where this rank holds rows
 * [rank*n_shard, (rank+1)*n_shard) of W (n_shard = its weight's n, equal on
 * every rank).  Computes the local slice, all-gathers the slices over NCCL and
 * leaves the full output on every rank.  y_full needs m*n_shard*nranks
 * elements of out_dtype; ws (scratch of the same size) may be NULL when
 * m == 1.  Runs on `stream` (a cudaStream_t; NULL = CUDA's default stream). */
int xq4_linear_sharded(xq4_comm *comm, const xq4_weight *w_shard,
                       const void *x_dev, void *y_full_dev, void *ws_dev,
                       int m, int out_dtype, void *stream);

/* xq4_linear_sharded with the all-gather fused into the GEMV: each rank's
 * kernel sends every output value it computes to every peer over NVLink, as
 * one 64-bit word (value and call number) in the peer's inbox, and copies
 * the peers' values for its own row range from its inbox into y_full, so
 * when the call's work on a rank's stream completes, that rank's y_full
 * (any device memory, m x n_total elements of out_dtype) holds every rank's
 * rows.  m in 1..15 and m x n_total <= XQ4_FUSED_MAX_VALUES; every rank
 * holds a shard of the same size and makes the same calls in the same
 * order.  The first call on a communicator allocates and maps the inboxes
 * (2 x XQ4_FUSED_MAX_VALUES x 8 bytes per rank, collective, device-wide
 * synchronising): make it before any stream capture.  A peer value that
 * does not arrive within 2 s sets fault bit 0x8 (xq4_device_fault), and
 * leaves the communicator unusable: the ranks' call counts are then out of
 * step, so the kernel that gave up marks the communicator on every rank.
 * From then on this rank's calls (and runs of chains with sharded ops on the
 * communicator) return XQ4_ETIMEDOUT; a peer's next call exchanges nothing
 * (its y_full holds its own rows only), sets fault bit 0x8 and marks it the
 * same way.  Destroy and re-create the communicator to go on.  Each CTA
 * waits for the matching CTA of every peer, so the whole grid must be
 * resident: XQ4_ENOTSUP when the device cannot hold it.  Do not run the call
 * beside other kernels that wait on peers.  Stands in for the column split
 * with a host gather of the per-column C sections (w4u_read_c,
 * crates/xnpu-cli/src/main.rs:3066-3091). */
#define XQ4_FUSED_MAX_VALUES (4u * 1024u * 1024u)
int xq4_linear_sharded_fused(xq4_comm *comm, const xq4_weight *w_shard, const void *x_dev,
                             void *y_full_dev, int m, int out_dtype, void *stream);

/* No counterpart in the reference.  xq4_linear_sharded without a workspace
 * and without allocating anything, for callers that cannot allocate device
 * memory when they run the op: a serving engine that reserved the GPU's
 * memory up front and refuses later allocations, a decode loop that cannot
 * afford cudaMalloc/cudaFree (cudaFree synchronises the device), or a
 * foreign-language caller with no device allocator.  For m > 1 the gather
 * stages through a fixed scratch array of XQ4_NOALLOC_SCRATCH_BYTES inside
 * the library; m * n_total * element size beyond that is rejected with
 * XQ4_EINVAL.  The array is committed on a device when the library's module
 * holding it is loaded there (CUDA loads modules lazily: at the first sharded
 * call on the device, or at this entry point's first call, whose set-up looks
 * up the array's device address), and stays until the process exits.  So
 * the entry point allocates nothing only after that set-up: a caller that
 * reserves the GPU's memory up front should make one call (m > 1) first, and
 * make it before any stream capture.  All calls share the array, so calls
 * that overlap on the GPU (other streams, other threads) race on it:
 * serialise them, for instance on one stream.  NCCL sets up a
 * communicator's connections, and allocates its own buffers, at the
 * communicator's first collective: run one collective on it (for instance
 * one xq4_linear_sharded call) before relying on this entry point to
 * allocate nothing. */
#define XQ4_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
int xq4_linear_sharded_noalloc(xq4_comm *comm, const xq4_weight *w_shard,
                               const void *x_dev, void *y_full_dev,
                               int m, int out_dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* XQ4_H */
