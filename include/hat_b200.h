/*
 * hat_b200.h — C ABI of the B200-native HAT super-resolution backend.
 *
 * This is the drop-in boundary for the GPU forward pass of hat-rs. Each entry point
 * replaces one piece of the reference's Rust interface; the comment on each names the
 * reference item (path within the hat-rs project, line numbers). Plain pointers and
 * sizes only; no ownership crosses the boundary except the opaque handle.
 *
 * Errors: every int-returning call returns 0 on success and a nonzero HAT_B200_E*
 * code on failure, writing a NUL-terminated message into `err` (when err != NULL and
 * errlen > 0). This replaces the reference's `Result<_, String>` (src/backend.rs:29-36).
 *
 * Threading: a handle is not thread-safe (the reference's `&mut self`,
 * src/gpu.rs:751-803). Use one handle per GPU, driven from any host thread, or one handle
 * over several GPUs (hat_b200_opts.ngpus), which runs one host thread per GPU inside each
 * forward call.
 */
#ifndef HAT_B200_H
#define HAT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HAT_B200_API __attribute__((visibility("default")))
#else
#define HAT_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define HAT_B200_OK 0
#define HAT_B200_EINVAL 1   /* bad argument or shape */
#define HAT_B200_EIO 2      /* checkpoint unreadable / malformed */
#define HAT_B200_ECUDA 3    /* a CUDA runtime error */
#define HAT_B200_ENOMEM 4   /* the memory guard refused the pass (src/memguard.rs:183-201) */
#define HAT_B200_ESELFTEST 5

/* Arithmetic mode. PARITY: fp32-accurate; every tensor-core operand is a hi/lo pair
 * carrying 22 significant bits and each product is three MMAs (hi*hi + hi*lo + lo*hi)
 * with fp32 accumulation, fp32 everywhere else; matches the reference's fp32 output to
 * <= 1e-4. The pairs are fp16 (kind::f16) when the embedding width is a multiple of 8,
 * else tf32 (kind::tf32); fp16 pairs cannot hold |x| >= 65504, and a pass that meets
 * such an operand is redone on tf32 pairs (see hat_b200_forward). FAST: single TF32
 * products on the tensor cores. */
#define HAT_B200_MODE_PARITY 0
#define HAT_B200_MODE_FAST 1
/* Kernel-level calls only: the CUDA-core fp32 kernels (the on-device cross-check). */
#define HAT_B200_MODE_SIMT 2

/* How a handle over several GPUs (hat_b200_opts.ngpus > 1) splits a forward call. BATCH:
 * the call's images are divided among the GPUs (contiguous, as equal as the count allows),
 * no communication between them. STRIP: every image is split into window-aligned row
 * strips, one per GPU, with the halo rows exchanged over NCCL before every layer that
 * reads across a strip edge and the channel-attention sums added across GPUs; the result
 * equals the one-GPU pass up to the order of those sums. */
#define HAT_B200_SHARD_BATCH 0
#define HAT_B200_SHARD_STRIP 1

typedef struct hat_b200 hat_b200;

/* Zero-initialise and set what is needed; the zero value of every field is its default. */
typedef struct hat_b200_opts {
    int device;      /* CUDA device ordinal this handle runs on (the first one when ngpus > 1) */
    int mode;        /* HAT_B200_MODE_* */
    int use_graph;   /* 1: capture each plan's launch sequence in a CUDA graph */
    int simt_only;   /* 1: CUDA-core fp32 kernels only (debug / cross-check path) */
    int ngpus;       /* 0 or 1: one GPU. N > 1: this handle drives N GPUs of this process,
                        one host thread each, and hat_b200_forward splits its work over them */
    const int* devices; /* the N device ordinals, or NULL for device, device + 1, ... */
    int shard;       /* HAT_B200_SHARD_*, for ngpus > 1 */
    int timeout_ms;  /* strip sharding: a call whose device work (which waits on the other
                        GPUs) has not finished after this long aborts the communicator and
                        returns HAT_B200_ECUDA instead of blocking; 0 = 120000 */
} hat_b200_opts;

/* What the checkpoint describes (src/weights.rs:28-57). */
typedef struct hat_b200_info {
    int scale, window, owin, embed, heads, head_dim, mlp_ratio, compressed, squeezed,
        head_feat, n_stages, n_blocks;
    float conv_scale, img_range, mean[3];
    char variant[32];
} hat_b200_info;

/* Gpu::new(&Weights) (src/gpu.rs:372-386) + Weights::load (src/weights.rs:60-129):
 * read and validate a checkpoint in the tools/convert.py safetensors layout, bring up
 * the device, check the weights fit (src/memguard.rs:211-225) and upload them. With
 * opts->ngpus > 1 this is done on every listed GPU, and in STRIP mode the GPUs are joined
 * in an NCCL communicator (no id from the caller). opts may be NULL (one GPU, device 0,
 * parity mode, CUDA graphs on). */
HAT_B200_API int hat_b200_create(const char* safetensors_path, const hat_b200_opts* opts,
                    hat_b200** out, char* err, size_t errlen);

/* Drop the handle and every device buffer it owns. */
HAT_B200_API void hat_b200_destroy(hat_b200* h);

HAT_B200_API int hat_b200_get_info(const hat_b200* h, hat_b200_info* out);

/* Backend::forward (src/backend.rs:29-36, src/gpu.rs:759-803): `in` is
 * [n][3][height][width] float32 in [0,1] on the HOST (not mean-adjusted); `out` is
 * [n][3][height*scale][width*scale] on the host after denormalisation. Pads to a
 * window multiple by edge replication (src/backend.rs:71-89) and crops after
 * (src/backend.rs:94-109). n = 1 is the reference's contract; n > 1 runs the images
 * back to back on this device. Blocks until `out` is written.
 * If an operand of the pass reaches fp16's range (|x| >= 65504), the whole call is redone:
 * with tf32 operand pairs when it was a GEMM operand (parity mode), and with the
 * attention on the fp32 CUDA-core kernels when it was q, k or v (any mode); the handle
 * keeps that setting for later calls (hat_b200_fp16_pairs then returns 0). A
 * strip-sharded handle returns HAT_B200_ECUDA instead.
 * On a handle over several GPUs the call is split as opts->shard says and returns once
 * every GPU's part is on the host; an error on any GPU fails the call (the message names
 * the GPU). */
HAT_B200_API int hat_b200_forward(hat_b200* h, int n, int height, int width, const float* in, float* out,
                     char* err, size_t errlen);

/* The same pass with `in`/`out` already in this device's memory, enqueued on `stream`
 * (a cudaStream_t, or NULL for the handle's own stream). Returns once enqueued; errors
 * the kernels find on the device (an expired wait, an operand beyond fp16's range; no
 * retry here) are reported by the next hat_b200_sync or hat_b200_forward. One-GPU
 * handles only (the buffers live on one device). */
HAT_B200_API int hat_b200_forward_device(hat_b200* h, int n, int height, int width, const float* d_in,
                            float* d_out, void* stream, char* err, size_t errlen);

/* Waits for the work this handle enqueued and returns HAT_B200_ECUDA with a message if a
 * kernel flagged an error since the last check (the reference's synchronous download
 * at the end of Gpu::forward, src/gpu.rs:799-802, is where its errors surface). */
HAT_B200_API int hat_b200_sync(hat_b200* h, char* err, size_t errlen);

/* 1 while the handle's parity-mode operands are fp16 pairs, 0 for tf32 pairs (always
 * for widths that are not a multiple of 8, and after a fallback) or another mode. */
HAT_B200_API int hat_b200_fp16_pairs(const hat_b200* h);

/* gpu::footprint_floats (src/gpu.rs:288-290) as bytes: the device bytes a pass at
 * this size allocates, computed without touching the device. */
HAT_B200_API size_t hat_b200_footprint_bytes(const hat_b200* h, int height, int width);

/* memguard::check_gpu (src/memguard.rs:183-201): 0 when a pass at this size fits the
 * free memory of the handle's device, HAT_B200_ENOMEM with the refusal text if not. */
HAT_B200_API int hat_b200_check_memory(const hat_b200* h, int height, int width, char* err, size_t errlen);

/* lightgpu::vm::free_vram (src/memguard.rs:174). */
HAT_B200_API int hat_b200_free_vram(int device, size_t* free_bytes, size_t* total_bytes);

/* vm::device() probe (src/main.rs:165-174): 1 if a CUDA device of compute
 * capability 10.x can be brought up, else 0. */
HAT_B200_API int hat_b200_probe(void);

/* --cuda-selftest (src/selftest.rs:437-523): every kernel against a host twin on
 * seeded inputs; the report goes to `log`. */
HAT_B200_API int hat_b200_selftest(int device, char* log, size_t loglen);

/* Weights::load + validate without a device (the --list-weights path, src/main.rs):
 * reads the checkpoint header and checks every tensor shape; fills `out`. */
HAT_B200_API int hat_b200_inspect(const char* safetensors_path, hat_b200_info* out, char* err, size_t errlen);

/* Kernel-level entry points (device pointers, enqueued on `stream`, NULL = default
 * stream), the units --cuda-selftest checks (src/cuda.rs:88-522 wrappers). */

/* y[m][n] = sum_k x[m][k] * w[n][k] + b[n]  (lg_linear / lg_conv1x1_rb, src/cuda.rs:162-169,440-453) */
HAT_B200_API int hat_b200_linear(int mode, const float* x, const float* w, const float* b, float* y,
                    int m, int n, int k, void* stream);

/* 3x3 conv, zero padding 1, on token-major [hgt][wid][cin] planes; w in PyTorch
 * [cout][cin][3][3] layout (lg_conv3x3_winograd, src/cuda.rs:88-106). */
HAT_B200_API int hat_b200_conv3x3(int mode, const float* x, const float* w, const float* b, float* y,
                     int hgt, int wid, int cin, int cout, void* stream);

/* Windowed multi-head attention of one HAB (hat_attention_d24/_d30, cuda/hat.cu:246-316
 * + hat_bias_gather + hat_mask_build): qkv is the token-major [hp][wp][3c] projection,
 * table the block's [(2win-1)^2][heads] bias table; shift 0 or win/2. */
HAT_B200_API int hat_b200_window_attention(int mode, const float* qkv, const float* table, float* out,
                              int hp, int wp, int c, int heads, int shift, void* stream);

/* The OCAB's overlapping attention (hat_unfold_kv, cuda/hat.cu:170-198, + attention):
 * 16x16 queries against the zero-padded 24x24 unfold of k and v. */
HAT_B200_API int hat_b200_overlap_attention(int mode, const float* qkv, const float* table, float* out,
                               int hp, int wp, int c, int heads, void* stream);

/* What a tiled pass did (src/tile.rs:29-43): the core side and margin used (window
 * multiples), the scale, the number of tiles and the largest sub-image a forward ran on. */
typedef struct hat_b200_tiling {
    int tile, margin, scale, tiles, largest_h, largest_w;
} hat_b200_tiling;

/* tile::forward (src/tile.rs:47-105), the `--tile` / `--mem` path: the image is cut into
 * window-aligned `tile`-pixel cores (rounded up to the window), each run as its own pass
 * on the core plus `margin` pixels of context (rounded up to the window, clamped to the
 * image, edge-replicated beyond it), and the cores are copied into `out` without
 * blending. Host buffers as hat_b200_forward; `info` may be NULL. The CLI's margin is two
 * windows (src/main.rs:303-305). Not available on a strip-sharded handle. */
HAT_B200_API int hat_b200_forward_tiled(hat_b200* h, int height, int width, const float* in, float* out, int tile,
                                        int margin, hat_b200_tiling* info, char* err, size_t errlen);

/* tile::auto_tile (src/tile.rs:147-184): the largest window-multiple core whose
 * sub-image (core + 2 * margin on a side) fits `budget_bytes` at `per_pixel_floats` floats
 * per pixel plus `constant_floats`, capped at the image. Returns HAT_B200_ENOMEM when not
 * even one window fits. No device needed. For `--mem`, per_pixel_floats is
 * hat_b200_footprint_bytes / 4 divided by the padded pixel count, and constant 0. */
HAT_B200_API int hat_b200_auto_tile(int height, int width, int window, uint64_t budget_bytes,
                                    uint64_t per_pixel_floats, uint64_t constant_floats, int margin, int* tile);

/* gpu_auto_tile (src/main.rs:107-140): the tile when neither --tile nor --mem is given,
 * halving from the larger image side until the memory guard admits a pass of that size
 * on the handle's device; *tile >= the larger side means the whole image fits. */
HAT_B200_API int hat_b200_gpu_auto_tile(const hat_b200* h, int height, int width, int* tile, char* err,
                                        size_t errlen);

/* Strip sharding of one large image over several GPUs (no counterpart in the reference,
 * which runs on one device). Padded rows are split into window-aligned strips
 * as equal as the 16-row windows allow (the first (hp/16) % nranks ranks take one window
 * row more); this writes rank `rank`'s padded rows [*r0, *r1) for an image `height`
 * rows high. No device needed. */
HAT_B200_API int hat_b200_strip_rows(int height, int nranks, int rank, int* r0, int* r1);

/* ncclGetUniqueId into `id` (idlen >= 128): rank 0 makes it, every rank passes the same
 * bytes to hat_b200_attach_strip. */
HAT_B200_API int hat_b200_nccl_unique_id(void* id, size_t idlen, char* err, size_t errlen);

/* Joins the handle to an NCCL communicator of `nranks` ranks (collective: every rank calls
 * it with the same id, one handle per GPU). From then on each forward computes only this
 * rank's row strip of the image: the input is the whole image on every rank, the output
 * buffer is the whole output and only this rank's rows of it are written (output rows
 * [scale*r0, scale*r1) cropped to the image). Halo rows are exchanged with the
 * neighbouring ranks before every layer that reads across the strip edge, and the
 * channel-attention means are summed over ranks; the result equals the unsharded pass up
 * to the order of those sums. Needs the tensor-core modes. */
HAT_B200_API int hat_b200_attach_strip(hat_b200* h, int rank, int nranks, const void* id, size_t idlen, char* err,
                                       size_t errlen);

/* hat_b200_linear without device allocation. No counterpart in the reference: it is for
 * callers that may not allocate device memory on this path (device memory already
 * reserved by another allocator, latency-critical loops, callers that must know the
 * call's device-memory use in advance).
 *
 * All scratch (the prepared weights, the tf32 hi/lo split of x in parity mode, and the
 * kernels' error word) lives in one statically allocated device array of
 * HAT_B200_NOALLOC_SCRATCH_BYTES per device; the call makes no cudaMalloc/cudaFree and
 * calls no allocating library routine. Sizes whose scratch exceeds the limit are refused
 * with HAT_B200_EINVAL and a message in `err` naming the bytes needed: about
 * 4*(n*k + 2*n_pad*k_pad + 2*m*k) + 256 bytes in parity mode, where n_pad and k_pad are
 * n and k rounded up to the tile sizes. The error word is zeroed by each call before its
 * first launch; everything else is rewritten before it is read.
 *
 * Each call looks up the array's address on the current device (cudaGetSymbolAddress,
 * which allocates nothing). The first call on a device also loads the library's device
 * code there; make that first call before any stream capture begins on the device.
 * Calls share the array: two calls in flight at once on the same device (from different
 * host threads) race on it and give wrong results, so serialise them. The call blocks
 * until its result is in `y`. Arguments otherwise as hat_b200_linear. */
#define HAT_B200_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
HAT_B200_API int hat_b200_linear_noalloc(int mode, const float* x, const float* w, const float* b, float* y,
                                         int m, int n, int k, void* stream, char* err, size_t errlen);

/* One eager pass at this size with a CUDA event between every launch, on the handle's
 * stream: per kind of kernel, its launch count, summed device time (ms) and the
 * algorithmic FLOPs and bytes of those launches, as a JSON object in `json`. (No
 * counterpart in the reference, which prints only the pass's wall time,
 * src/main.rs:285-288.) */
HAT_B200_API int hat_b200_profile(hat_b200* h, int height, int width, char* json, size_t jsonlen,
                                  char* err, size_t errlen);

/* PNG file I/O around the forward pass (src/image.rs). Decoding accepts 8- and 16-bit grey,
 * grey + alpha, RGB and RGBA, interlaced or not (indexed colour and other bit depths are
 * refused as the reference refuses them); the output is planar [3][height][width] float
 * in [0, 1], grey replicated to three channels and alpha dropped.
 *
 * image::load_rgb (src/image.rs:43-96): decodes the file at `path` into `out` (capacity
 * `out_floats`; pass NULL / 0 to learn the size first) and sets *width, *height.
 * HAT_B200_EIO for unreadable or malformed files, HAT_B200_EINVAL when `out` is too small. */
HAT_B200_API int hat_b200_png_load(const char* path, float* out, size_t out_floats, int* width, int* height,
                                   char* err, size_t errlen);

/* image::load_rgb_stream (src/image.rs:49-96): the same decode from `len` bytes in memory
 * (the CLI's `-i -`). */
HAT_B200_API int hat_b200_png_decode(const uint8_t* bytes, size_t len, float* out, size_t out_floats, int* width,
                                     int* height, char* err, size_t errlen);

/* Image::to_rgb8 (src/image.rs:29-39): planar [3][height][width] float to interleaved
 * 8-bit RGB, clamped to [0, 1], times 255, rounded half up. */
HAT_B200_API int hat_b200_to_rgb8(const float* planar, int width, int height, uint8_t* rgb);

/* image::save_rgb (src/image.rs:99-106): writes 8-bit RGB (interleaved, `width` x `height`)
 * as a PNG file. */
HAT_B200_API int hat_b200_png_save(const char* path, int width, int height, const uint8_t* rgb, char* err,
                                   size_t errlen);

/* image::save_rgb_stream (src/image.rs:108-114): the same encode into `out` (capacity
 * `cap` bytes); *len is set to the encoded size, and HAT_B200_EINVAL is returned (with
 * *len set) when `cap` is too small. */
HAT_B200_API int hat_b200_png_encode(int width, int height, const uint8_t* rgb, uint8_t* out, size_t cap, size_t* len,
                                     char* err, size_t errlen);

/* Sets the deadline of a strip-sharded call's device work (hat_b200_opts.timeout_ms) on every
 * GPU of the handle; ms <= 0 restores the default (120000). A first call, which also sets up the
 * NCCL connections and may find its peers still starting, can run under a longer deadline than
 * the calls after it. (No counterpart in the reference, which runs on one device.) */
HAT_B200_API int hat_b200_set_timeout(hat_b200* h, int ms);

/* The GPUs this handle drives (1 unless created with ngpus > 1). */
HAT_B200_API int hat_b200_gpu_count(const hat_b200* h);

/* Kernel launches issued by this handle since creation, over all its GPUs
 * (src/cuda.rs:542-555). */
HAT_B200_API uint64_t hat_b200_launch_count(const hat_b200* h);

#ifdef __cplusplus
}
#endif
#endif
