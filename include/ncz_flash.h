/*
 * ncz_flash.h -- C ABI of the B200 (sm_100a) flash-attention forward library
 * (libncz_flash.so).  It is a drop-in for the `flash` module of not-cute-zig.
 *
 * All pointers passed to the launch entry points are DEVICE pointers owned by
 * the caller; the library never frees them.  Launches are asynchronous on the
 * given stream (NULL = the legacy default stream).  Validation happens before
 * any launch, and nothing is launched when it fails.  No function prints.
 *
 * Tensor layout (the reference's, src/flash.zig:5-15): Q/K/V are f16, O is f32
 * (f16 optional through ncz_flash_fwd_ex).  batch_heads independent slices
 * start at slice * *_stride elements; inside a slice, row r starts at
 * r * row_stride elements, where row_stride is head_dim in the reference API.
 */
#ifndef NCZ_FLASH_H
#define NCZ_FLASH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes.  0..15 mirror the reference's CudaError set one to one
 * (src/cuda.zig:134-151, mapping at src/cuda.zig:160-177).  16..17 are new:
 * a bounded in-kernel wait expired, and an alignment the chosen path needs is
 * missing (only returned when a caller forces the TMA path). */
typedef enum ncz_status {
    NCZ_SUCCESS = 0,
    NCZ_ERROR_OUT_OF_MEMORY = 1,
    NCZ_ERROR_OVERFLOW = 2,
    NCZ_ERROR_SHARED_OBJECT_INIT_FAILED = 3,
    NCZ_ERROR_NOT_FOUND = 4,
    NCZ_ERROR_INVALID_VALUE = 5,
    NCZ_ERROR_INVALID_CONTEXT = 6,
    NCZ_ERROR_INVALID_DEVICE = 7,
    NCZ_ERROR_INVALID_IMAGE = 8,
    NCZ_ERROR_CONTEXT_IS_DESTROYED = 9,
    NCZ_ERROR_LAUNCH_FAILED = 10,
    NCZ_ERROR_LAUNCH_OUT_OF_RESOURCES = 11,
    NCZ_ERROR_LAUNCH_TIMEOUT = 12,
    NCZ_ERROR_ILLEGAL_ADDRESS = 13,
    NCZ_ERROR_NO_DEVICE = 14,
    NCZ_ERROR_NOT_INITIALIZED = 15,
    NCZ_ERROR_UNKNOWN = 16,
    NCZ_ERROR_DEVICE_TIMEOUT = 17,
    NCZ_ERROR_MISALIGNED = 18
} ncz_status;

/* Element types: O is f32, f16 or bf16; Q/K/V are f16 or bf16.  With bf16
 * inputs P is rounded to bf16 before PV (a tensor-core MMA takes A and B of one
 * type). */
typedef enum ncz_dtype { NCZ_DTYPE_F32 = 0, NCZ_DTYPE_F16 = 1, NCZ_DTYPE_BF16 = 2 } ncz_dtype;

/* Producer selection: AUTO picks the TMA path when every Q/K/V base pointer is
 * 16-byte aligned and every Q/K/V stride is a multiple of 8 elements, and the
 * load/store-unit (LSU) path otherwise.  Both are the same sm_100a kernel
 * (tcgen05 MMAs, TMEM accumulators); they differ only in how K/V/Q tiles
 * reach shared memory. */
typedef enum ncz_producer {
    NCZ_PRODUCER_AUTO = 0,
    NCZ_PRODUCER_TMA = 1,
    NCZ_PRODUCER_LSU = 2
} ncz_producer;

/* Extended descriptor (ncz_flash_fwd_ex).  Zero row strides mean head_dim
 * (the reference layout).  Fields mirror flash.Options (src/flash.zig:5-15)
 * plus: per-row strides, O element type, producer override, device ordinal
 * (-1 = current device) and stream. */
typedef struct ncz_flash_desc {
    const void *q;
    const void *k;
    const void *v;
    void *o;
    size_t batch_heads;
    size_t seq_len;
    size_t head_dim;
    size_t q_stride, k_stride, v_stride, o_stride;                 /* per slice, elements */
    size_t q_row_stride, k_row_stride, v_row_stride, o_row_stride; /* per row, 0 = head_dim */
    float scale;
    uint32_t causal;
    int32_t o_dtype;  /* ncz_dtype */
    int32_t producer; /* ncz_producer */
    int32_t device;   /* CUDA ordinal, -1 = current */
    void *stream;     /* cudaStream_t / CUstream, NULL = default stream */
    int32_t in_dtype; /* Q/K/V type: NCZ_DTYPE_F16 (or 0) or NCZ_DTYPE_BF16 */
} ncz_flash_desc;

/* Loads nothing eagerly; resolves the driver entry points and records the
 * device count.  Idempotent.  Called implicitly by every launch. */
int ncz_init(void);
/* Releases what the library owns on every device (split-KV memory pools,
 * host-pipeline streams and events) and drops its cached per-device state
 * (initialisation, kernel attributes, tensor maps, SM counts); the next call
 * initialises again.  Kernels and copies in flight are not waited for: the
 * runtime frees a stream or pool once its work is done.  Returns the first
 * error of the release, else NCZ_SUCCESS.  No other thread may be inside the
 * library meanwhile. */
int ncz_shutdown(void);

/* flash.Options.validate (src/flash.zig:16-28): batch_heads > 0, seq_len > 0,
 * head_dim in {16,32,64}, every slice stride >= seq_len * head_dim. */
int ncz_flash_validate(size_t batch_heads, size_t seq_len, size_t head_dim, size_t q_stride,
                       size_t k_stride, size_t v_stride, size_t o_stride);

/* Validation of the extended descriptor: the reference rules with row strides
 * (each row stride >= head_dim, each slice stride >= (seq_len-1)*row_stride +
 * head_dim), o_dtype and producer in range. */
int ncz_flash_validate_ex(const ncz_flash_desc *desc);

/* flash.selectKernel (src/flash.zig:72-96).  Writes the kernel label
 * ("flash_fwd_sm100a_d16", "_d32" or "_d64") into `label` (NUL-terminated,
 * truncated to `cap`) and the threads per CTA into *threads.  One sm_100a
 * kernel family replaces flash_attention_fwd_{opt,v2,h64,h64_bn32,h64_causal};
 * ncz_flash_fwd_named accepts those names and these labels. */
int ncz_flash_select(size_t batch_heads, size_t seq_len, size_t head_dim, uint32_t causal,
                     char *label, size_t cap, uint32_t *threads);

/* The reference kernel argument tuple (src/flash.zig:55-68, the 12 arguments
 * of flash_attention_fwd_* plus batch_heads and a stream).  Replaces
 * selectKernel + Function.launch (src/main.zig:820-852, :1022-1035) and the
 * exported kernel symbols (src/main_device.zig:19-47).  Q/K/V f16, O f32. */
int ncz_flash_fwd(const void *q, const void *k, const void *v, void *o, size_t batch_heads,
                  size_t seq_len, size_t head_dim, size_t q_stride, size_t k_stride,
                  size_t v_stride, size_t o_stride, float scale, uint32_t causal, void *stream);

/* module.getFunction(name) + Function.launch(cfg, tuple) of the reference's
 * callers (src/main.zig:93-94, :820-852): launches the kernel named `kernel`
 * with the 12-argument tuple and batch_heads (grid.y).  Accepted names are the
 * reference's exported flash kernels and this library's labels:
 *   flash_attention_fwd          d 16/32/64          src/kernels.zig:380-394
 *   flash_attention_fwd_opt      d 16/32/64          src/flash_opt.zig:17-31
 *   flash_attention_fwd_v2       d 16/32/64          src/flash_v2.zig:23-37
 *   flash_attention_fwd_h64      d 64                src/flash_h64.zig:21-35
 *   flash_attention_fwd_h64_bn32 d 64                src/flash_h64_bn32.zig:26-40
 *   flash_attention_fwd_h64_causal d 64, always causal (ignores `causal`)
 *                                                    src/flash_h64_causal.zig:20-35
 *   flash_fwd_sm100a_d16 / _d32 / _d64  that head_dim only
 * As each of those kernels does, a call with seq_len 0 or a head_dim the name
 * does not accept returns NCZ_SUCCESS without launching or writing O.  Any
 * other name is NCZ_ERROR_NOT_FOUND (cuModuleGetFunction's answer);
 * batch_heads 0 is NCZ_ERROR_INVALID_VALUE (a launch with grid.y 0).  The
 * reference kernels check no strides; here they are validated as in
 * ncz_flash_fwd. */
int ncz_flash_fwd_named(const char *kernel, const void *q, const void *k, const void *v, void *o,
                        size_t batch_heads, size_t seq_len, size_t head_dim, size_t q_stride,
                        size_t k_stride, size_t v_stride, size_t o_stride, float scale, uint32_t causal,
                        void *stream);

/* Head dimensions (bit 0: 16, bit 1: 32, bit 2: 64) and forced causality
 * (1 = always causal) of a kernel name accepted by ncz_flash_fwd_named;
 * NCZ_ERROR_NOT_FOUND for any other name. */
int ncz_flash_kernel_info(const char *kernel, uint32_t *head_dims, uint32_t *always_causal);

/* flash.launch (src/flash.zig:31-70): like ncz_flash_fwd, but takes the
 * slice lengths (elements) so requireLen (src/flash.zig:98-100) is checked:
 * each length must be >= batch_heads * stride. */
int ncz_flash_launch(const void *q, size_t q_len, const void *k, size_t k_len, const void *v,
                     size_t v_len, void *o, size_t o_len, size_t batch_heads, size_t seq_len,
                     size_t head_dim, size_t q_stride, size_t k_stride, size_t v_stride,
                     size_t o_stride, float scale, uint32_t causal, void *stream);

/* Extended launch: row strides, f16 O, producer override, device ordinal.
 * No reference counterpart beyond flash.launch (src/flash.zig:31-70). */
int ncz_flash_fwd_ex(const ncz_flash_desc *desc);

/* Extended launch with an explicit split-KV request.  splits = 0 chooses
 * automatically (what every other launch entry point does: split when the
 * grid of batch_heads x ceil(seq_len/256) CTAs fills at most half the SMs),
 * 1 never splits, n > 1 splits each Q group's K tiles into up to min(n, 8) ranges
 * computed by separate CTAs and merged by a second kernel.  Partial results
 * live in a library-owned stream-ordered memory pool; nothing is allocated
 * when no split is made.  The reference has no split path (its grid is
 * (ceil(S/16), bh), src/flash.zig:45-69). */
int ncz_flash_fwd_splits(const ncz_flash_desc *desc, int splits);

/* Bytes of the fixed split-KV scratch that ncz_flash_fwd_static uses on each
 * device (held from library load until the process exits). */
#define NCZ_STATIC_SCRATCH_BYTES (16u << 20)

/* ncz_flash_fwd_splits for callers that must not let this library allocate
 * device memory: hosts whose own allocator owns every device buffer (as the
 * reference's Zig host does with cuda.malloc), and request loops that cannot
 * afford an allocation that may block, or fail mid-request when memory is
 * tight.  No counterpart in the reference, whose kernels need no scratch.
 *
 * The split-KV partials (splits x batch_heads x seq_len x (head_dim + 2)
 * floats) go to a fixed array of NCZ_STATIC_SCRATCH_BYTES in the library's
 * device image instead of the memory pool; nothing is allocated or freed.
 * splits = 0 (automatic) takes the largest split count whose partials fit,
 * down to no split.  An explicit splits > 1 whose partials do not fit returns
 * NCZ_ERROR_OUT_OF_MEMORY before anything is launched.  The first call on a
 * device looks up the array's device address (device switched to desc->device
 * for it), so make that first call before any stream capture.  Every call on a
 * device shares the one array, which keeps the last call's partials (each call
 * writes every partial it reads, so nothing needs clearing): calls whose
 * kernels overlap on the GPU race, so order them (one stream, or streams
 * ordered by events).  ncz_flash_fwd_splits has no such restriction. */
int ncz_flash_fwd_static(const ncz_flash_desc *desc, int splits);

/* One call, several devices: descs[i] is launched on descs[i].device (each on
 * its own stream); the caller's current device is restored.  Used to shard
 * batch x head slices across GPUs.  The reference has one device only
 * (src/cuda.zig:181-196); this replaces a per-device loop over flash.launch. */
int ncz_flash_fwd_multi(const ncz_flash_desc *descs, int count);

/* Host-buffer forward with overlapped copies.  q_host, k_host, v_host and
 * o_host are HOST buffers laid out exactly like desc->q/k/v/o (same strides);
 * desc->q/k/v/o are caller-owned device buffers of the same layout that stage
 * them.  Slices are processed in chunks of chunk_slices (0 = bh/8 rounded up,
 * but at least 4 MiB of Q/K/V per chunk, the first two and last two chunks a
 * quarter and a half of that):
 * a chunk's Q/K/V upload, its forward and its O download run on separate
 * streams, so the upload of chunk i+1 overlaps the forward of chunk i and the
 * download of chunk i-1.  Host buffers must be page-locked (pinned) for the
 * copies to run asynchronously.  Everything is ordered on desc->stream: work
 * enqueued on it afterwards runs once O is in host memory.  Each chunk of O
 * comes back as one contiguous range, from its first slice's first element to
 * its last slice's last active element: where O has padding (o_row_stride >
 * head_dim, or slices more than a slice apart) the host padding inside that
 * range receives whatever the device O buffer holds there, which the kernel
 * never writes.  The device entry points leave O padding untouched.  Replaces the
 * upload / flash.launch / download sequence of the reference's callers
 * (src/main.zig:254-271). */
int ncz_flash_fwd_host(const ncz_flash_desc *desc, const void *q_host, const void *k_host,
                       const void *v_host, void *o_host, size_t chunk_slices);

/* Synchronises `stream` (on `device`, -1 = current), then reads and clears the
 * device's in-kernel status word.  Returns NCZ_ERROR_DEVICE_TIMEOUT when a
 * bounded wait expired in a kernel since the last call, a CUDA error code
 * when the stream faulted, NCZ_SUCCESS otherwise.  *detail (may be NULL)
 * receives the raw status word (0 if clean). */
int ncz_flash_sync_status(int device, void *stream, uint32_t *detail);

/* --- Test hooks for the failure-detection path (device work, no fault). --- */

/* Test hook: the split-KV plan of a launch (host only, no GPU): requested 0 =
 * automatic on `sms` SMs, 1 = none, n = up to n ranges; out[0] = ranges,
 * out[1] = K tiles per range. */
int ncz_test_split_plan(size_t batch_heads, size_t seq_len, int requested, size_t sms, int32_t *out);

/* Test hook: the slice chunks of ncz_flash_fwd_host for a chunk size (taper =
 * the tapered first and last chunks of the default plan); *count = chunks,
 * out[0 .. count) their slice counts (NCZ_ERROR_OVERFLOW when cap is short). */
int ncz_test_chunk_plan(size_t batch_heads, size_t chunk_slices, int taper, size_t *out, size_t cap, size_t *count);

/* Test hook: the work item `item` of a launch with this shape, split count
 * (as ncz_flash_fwd_splits; 1 = none) and chunk of slices in the item order:
 * out[0..7] = slice, first Q row, split, first K tile, K tiles of Q tile 0,
 * of Q tile 1, their maximum, and the resolved split count.  Host only; no
 * GPU needed.  NCZ_ERROR_INVALID_VALUE for an item outside the launch. */
int ncz_test_item_work(size_t batch_heads, size_t seq_len, uint32_t causal, int splits, int chunk_slices, int item,
                       int32_t *out);

/* Test hook: the work item `item` of a launch whose top `split_groups` groups
 * of two 128-row Q tiles (1 .. all of them; the heaviest under causal
 * masking) run as split-Q items: one Q tile per item, its K tiles alternating
 * between the CTA's two pipelines.  Those come first in each chunk of
 * `chunk_slices` slices, heaviest Q tile first, then the other groups' items
 * of two Q tiles, heaviest group first.  out[0..5] = slice, first Q row, K
 * tiles of slot 0, of slot 1, the item's K tiles, K tile stride (2 for a
 * split-Q item, 1 otherwise).  Host only; NCZ_ERROR_INVALID_VALUE past the
 * launch. */
int ncz_test_qsplit_work(size_t batch_heads, size_t seq_len, uint32_t causal, int chunk_slices, int split_groups,
                         int item, int32_t *out);

/* Test hook: the split-Q plan of a launch without split-KV on `sms` SMs:
 * out[0] = groups run as split-Q items (all of them when the items of two Q
 * tiles number fewer than 1.25 per SM, else 0), out[1] = the launch's work
 * items.  Host only. */
int ncz_test_qsplit_plan(size_t batch_heads, size_t seq_len, size_t sms, int32_t *out);

/* Test hook: the split-Q choice of every following launch of this process:
 * 0 automatic (the default), 1 whenever the launch has no split-KV, 2 never.
 * Results agree either way within the parity bound; the hook lets tests run
 * both item kinds on the same shape. */
int ncz_test_set_qsplit(int mode);

/* groups >= 0: every following launch without split-KV runs the Q tiles of
 * its top `groups` Q-tile groups (clamped to the launch's groups) as split-Q
 * items and the rest as items of two Q tiles, whatever ncz_test_set_qsplit
 * chose; -1 (the default) hands the choice back to that mode.  Tests and
 * timing sweeps use it to run one shape under every mix of item kinds. */
int ncz_test_set_qsplit_groups(int groups);

/* Twin items: a launch with seq_len <= 128 (one Q tile per slice) and no
 * split-KV runs items of two slices, one per pipeline, unless a test forces
 * split-Q items.  enable = 1 (the default) allows them, 0 runs items of one
 * slice; results are bit-identical either way. */
int ncz_test_set_twin(int enable);

/* Test hook: out[0] = rows per Q tile (128), out[1] = keys per K/V tile (64):
 * the units of the item-order and split-plan hooks' tile counts. */
int ncz_test_tile_shape(int32_t *out);

/* Test hook: twin item `item` of a launch of batch_heads slices of seq_len <=
 * 128: out[0], out[1] = the slices of slots 0 and 1 (-1 when slot 1 is empty),
 * out[2], out[3] = their K tiles, out[4] = ring tiles of the item, out[5],
 * out[6] = the slices of ring tiles 0 and 1 (-1 when absent), out[7] = the
 * item kind (2 = twin; 0 = one slice, the last item of an odd count).  Host
 * only. */
int ncz_test_twin_work(size_t batch_heads, size_t seq_len, uint32_t causal, int item, int32_t *out);

/* Bound of every in-kernel mbarrier wait on `device` (-1 = current), in SM
 * cycles; 0 restores the default (4e9, about 2 s).  A test shortens it so an
 * expired wait is seen quickly. */
int ncz_test_set_wait_limit(int device, uint64_t cycles);

/* enable != 0: in every following launch on `device`, the MMA warp of the
 * first Q tile never signals its first scores, so that tile's softmax wait
 * runs out, the CTA aborts cleanly and ncz_flash_sync_status reports
 * NCZ_ERROR_DEVICE_TIMEOUT.  enable = 0 restores normal operation. */
int ncz_test_drop_arrive(int device, int enable);

/* Human-readable name of a status code (static storage). */
const char *ncz_status_string(int status);

/* Number of kernel launches this library has issued in this process
 * (all devices).  Used by benchmarks to report their own launch count. */
uint64_t ncz_launch_count(void);

/* --- Host-side helpers used by unit tests (no device work). --- */

/* tcgen05 shared-memory matrix descriptor (64-bit) for a tile at shared
 * address `smem_addr`: layout_type is the UMMA swizzle code (0 none, 2 =
 * 128B, 4 = 64B, 6 = 32B); lbo/sbo in bytes.  Extends the warp-MMA
 * Descriptor of src/mma.zig:23-57 to the sm_100 shared-memory descriptor. */
uint64_t ncz_umma_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                            uint32_t layout_type);

/* tcgen05 kind::f16 instruction descriptor: f16 A/B, f32 accumulate, given
 * M, N and operand majors (0 = K-major, 1 = MN-major). */
uint32_t ncz_umma_instr_desc_f16(uint32_t m, uint32_t n, uint32_t a_major, uint32_t b_major);
/* The same with bf16 A and B (bits 7..9 and 10..12 = 1). */
uint32_t ncz_umma_instr_desc_bf16(uint32_t m, uint32_t n, uint32_t a_major, uint32_t b_major);

/* Byte-address swizzle of a TMA SWIZZLE_{32,64,128}B tile: the shared-memory
 * byte offset at which logical byte offset `offset` of a tile with
 * `span_bytes` (32, 64 or 128) wide rows is stored.  Generalises
 * layout.XorSwizzle (src/layout.zig:327-358) from element to byte offsets. */
uint32_t ncz_tma_swizzle_offset(uint32_t span_bytes, uint32_t offset);

#ifdef __cplusplus
}
#endif

#endif /* NCZ_FLASH_H */
