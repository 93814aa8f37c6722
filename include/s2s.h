/* s2s.h - C ABI of the B200-native Swin2SR forward pass.
 *
 * This is the boundary the reference's GPU backend plugs into: swin2sr-rs
 * src/gpu.rs implements `Backend` (src/backend.rs:29-49) for `Gpu`; a drop-in
 * `Gpu` keeps that trait impl and forwards to these entry points through an FFI
 * binding. Plain C types only; every pointer is caller-owned unless stated.
 *
 * Threading: a handle is not thread-safe (the reference's `forward` takes
 * `&mut self`); one CUDA stream per handle; the host-buffer calls return when the
 * result is on the host. Calls on one handle from several threads (only the
 * allocation-free attention entry point below invites that) share its kernel
 * launch counter, which is atomic, and its last-error string, which holds the
 * message of whichever call failed last.
 */
#ifndef S2S_H
#define S2S_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference reports errors as `Result<_, String>` and its CLI
 * retries with a smaller tile only when the message contains "OUT_OF_MEMORY"
 * (src/main.rs:660-662): S2S_ERR_OOM's message always contains
 * "CUDA_ERROR_OUT_OF_MEMORY" so that retry keeps working. */
enum {
  S2S_OK = 0,
  S2S_ERR_OOM = 1,         /* device allocation failed */
  S2S_ERR_INVALID = 2,     /* bad argument, shape or missing tensor */
  S2S_ERR_CUDA = 3,        /* any other CUDA error */
  S2S_ERR_NCCL = 4,        /* collective failure (sharded modes) */
  S2S_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up */
  S2S_ERR_UNSUPPORTED = 6, /* architecture this build does not implement */
  S2S_ERR_SELFTEST = 7     /* s2s_selftest: a consistency check failed (see its report) */
};

/* Reconstruction heads (src/weights.rs:18-29, Upsampler). */
enum {
  S2S_PIXELSHUFFLE = 0,
  S2S_PIXELSHUFFLEDIRECT = 1,
  S2S_NEARESTCONV = 2,
  S2S_PIXELSHUFFLE_AUX = 3
};

/* The architecture, as the checkpoint's __metadata__ states it
 * (src/weights.rs:94-137; tools/convert.py:224-236). */
typedef struct s2s_config {
  int upsampler;     /* S2S_PIXELSHUFFLE ... */
  int scale;         /* 2 or 4 */
  int window;        /* 8 */
  int embed;         /* 60 or 180 */
  int heads;         /* attention heads per block */
  int mlp_ratio;     /* 2 */
  int n_depths;      /* RSTB stages */
  int depths[16];    /* blocks per stage */
  float img_range;   /* 1.0 */
  float mean[3];     /* RGB mean subtracted before the network */
} s2s_config;

/* One converted-checkpoint tensor, row-major fp32, borrowed for the call only
 * (the reference hands out `&[f32]` views of its mmap, src/weights.rs:240-242).
 * Names are tools/convert.py's: "layers.{s}.residual_group.blocks.{b}.attn.qkv.wq",
 * ".attn.cpb_pre", "conv_first.weight", ... */
typedef struct s2s_tensor {
  const char* name;
  const float* data;
  int ndim;
  int64_t shape[4];
} s2s_tensor;

typedef struct s2s_handle s2s_handle;

/* Gpu::new (src/gpu.rs:101-125): validate, repack every needed tensor to the
 * device layouts (fp16 K-major GEMM operands, fp32 biases / norms / bias table)
 * and upload them once. `device` is the CUDA ordinal. On failure *out is NULL
 * and the message is available from s2s_last_error(NULL). */
int s2s_create(const s2s_config* cfg, const s2s_tensor* tensors, int n_tensors, int device,
               s2s_handle** out);

/* Backend::forward (src/backend.rs:34; src/gpu.rs:741-754): `in_chw` is
 * [3][h][w] fp32 ALREADY mean-adjusted by Pre::adjust (src/backend.rs:76-86) and
 * unpadded; the library pads (src/plan.rs:116-139), runs the network and writes
 * `out_chw` = [3][h*scale][w*scale], denormalised and cropped, not clamped
 * (src/cpu.rs:1925-1941). `aux_chw` may be NULL; for the pixelshuffle_aux head it
 * receives [3][hp][wp] (s2s_aux_dims), denormalised and NOT cropped
 * (src/cpu.rs:1892-1903). Host buffers; synchronous. */
int s2s_forward(s2s_handle* h, int height, int width, const float* in_chw, float* out_chw,
                float* aux_chw);

/* The same for `batch` independent images of one size, contiguous
 * [batch][3][h][w] -> [batch][3][h*s][w*s] (+ [batch][3][hp][wp] aux). */
int s2s_forward_batch(s2s_handle* h, int batch, int height, int width, const float* in,
                      float* out, float* aux);

/* Device-resident variant: pointers are device memory on the handle's device,
 * work is enqueued on `stream` (a cudaStream_t; NULL = the handle's own stream)
 * and the call returns without synchronising. */
int s2s_forward_device(s2s_handle* h, int batch, int height, int width, const float* d_in,
                       float* d_out, float* d_aux, void* stream);

/* Backend::aux geometry: the padded plane of an h x w input (src/plan.rs:39-47).
 * Returns S2S_ERR_INVALID for heads without an aux image. */
int s2s_aux_dims(const s2s_handle* h, int height, int width, int* aux_h, int* aux_w);

/* gpu::uploaded_bytes (src/gpu.rs:792-799): device bytes held by the weights. */
int64_t s2s_uploaded_bytes(const s2s_handle* h);

/* per_pixel_floats(gpu = true) (src/backend.rs:300-383), made exact: the
 * activation bytes a forward of `batch` h x w images allocates. */
int64_t s2s_workspace_bytes(const s2s_handle* h, int batch, int height, int width);

/* The last error message of `h` (or, when h is NULL, of the last failed s2s_create
 * or handle-less call on this thread). */
const char* s2s_last_error(const s2s_handle* h);

/* Per-launch CUDA-event timing, the SWIN2SR_PROFILE_GPU profiler
 * (src/cuda.rs:109-140, 163-259). The environment variable turns it on at
 * create time; this toggles it at run time. Events are recorded on the stream
 * each kernel is launched on. `only` (may be NULL) restricts timing to kernel
 * classes whose name starts with it, so a timed run pays for two events per
 * launch of that class only. */
int s2s_profile_enable(s2s_handle* h, int on, const char* only);

/* Aggregated profile since the last reset, one line per kernel class:
 * "name launches total_ms". Writes at most `cap` bytes (NUL-terminated) and
 * returns the length needed. Resets the counters when `reset` is non-zero. */
int s2s_profile_report(s2s_handle* h, char* buf, int cap, int reset);

/* Kernel launches enqueued by this handle since creation. */
int64_t s2s_launch_count(const s2s_handle* h);

/* Diagnostics (the counterpart of the reference's `dump` hooks, src/cpu.rs:1405,
 * 1453-1459, which name every activation for bisection against the torch
 * network): stop the next forwards after `launches` kernel launches (-1 = run
 * to the end), and read a named workspace buffer of the current plan back as
 * fp32 ("P", "F0", "F0h", "X", "X16", "S", "QKV", "AO", "H16",
 * "HA", "HB0", "HB1", "HB2", "BIC", "BICF", "AUXRAW"). s2s_debug_read returns
 * the element count, or -1 for an unknown name / no plan. */
int s2s_debug_stop_after(s2s_handle* h, int64_t launches);
int64_t s2s_debug_read(s2s_handle* h, const char* buffer, float* host, int64_t capacity);

/* Diagnostics of the peer-store halo transport on one GPU (no counterpart in the
 * reference): two exchanges of `rows` rows (1..8) on a scratch band plane whose
 * neighbours on both sides are the plane itself, through the kernel, flags and
 * epochs a sharded forward uses - its last rows must land in its top halo and its
 * first rows in its bottom halo. With `missing` != 0 the neighbours' mailbox is one
 * that no kernel serves, so the exchange's waits run out after about a second:
 * S2S_ERR_TIMEOUT, and the handle stays usable. */
int s2s_debug_halo_loopback(s2s_handle* h, int rows, int missing);

/* ---- Row-band sharding of one image across GPUs. No counterpart in the
 * reference, which runs an image on one GPU (src/gpu.rs:462-583 is the forward
 * each band repeats). The padded plane's window rows are split into contiguous
 * bands, one per rank (one process per GPU); each rank runs the whole network on
 * its band and swaps halo rows with its neighbours by NCCL point-to-point: 4 rows
 * (cyclically) before every shifted block, 1 row before every 3x3 convolution, 4
 * rows before the head. The output equals the whole-image forward's, split by rows:
 * rank r produces output rows [row0 * scale, row1 * scale) (s2s_band_rows). */
#define S2S_BAND_ID_BYTES 128

/* The communicator id: made on one rank, its S2S_BAND_ID_BYTES bytes handed to the
 * others by the caller (any channel). S2S_ERR_NCCL when libnccl.so.2 is absent. */
int s2s_band_unique_id(void* id, int cap);

/* Make `h` rank `rank` of `world` bands (collective: every rank calls it with the
 * same id). world == 1 leaves band mode. Afterwards only the s2s_forward_band*
 * calls run forwards on `h`. S2S_ERR_UNSUPPORTED for the pixelshuffle_aux head. */
int s2s_band_init(s2s_handle* h, int rank, int world, const void* id, int id_bytes);

/* The same for `world` handles of this process (one host thread per handle runs
 * s2s_forward_band* concurrently; halos move by device-to-device copies). */
int s2s_band_init_local(s2s_handle** handles, int world);

/* Input rows [row0, row1) of a `height`-row image whose output this rank produces. */
int s2s_band_rows(const s2s_handle* h, int height, int* row0, int* row1);

/* One image, every rank at once: d_in is the whole [3][h][w] input (device), d_out
 * this rank's [3][(row1 - row0) * s][w * s] output rows (device); enqueued on
 * `stream` (NULL = the handle's) without synchronising. */
int s2s_forward_band(s2s_handle* h, int height, int width, const float* d_in, float* d_out,
                     void* stream);
/* Host-buffer variant (synchronous). */
int s2s_forward_band_host(s2s_handle* h, int height, int width, const float* in, float* out);

/* Host-only helpers (no device, no handle): the split of `window_rows` among
 * `world` bands (rank's window rows [w0, w1)), and the transfers of one halo
 * exchange of `rows` rows in issue order, 4 ints each (0 send / 1 receive, peer,
 * first local row, rows; the band's own rows are local [8, 8 + own_rows)). The
 * latter returns the count, or -1 for bad arguments. */
int s2s_band_partition(int window_rows, int world, int rank, int* w0, int* w1);
int s2s_band_halo_ops(int rank, int world, int own_rows, int rows, int cyclic, int* ops, int cap);

/* No counterpart in the reference. Window attention of block `block` of stage
 * `stage` for callers that must not allocate: it allocates no device or host
 * memory and needs no plan. The window -> image row table it reads (which a
 * forward keeps in its workspace) lives in a fixed device array of the library
 * holding S2S_NOALLOC_MAX_TOKENS rows (4 MiB); batch * hp * wp above that is
 * rejected with S2S_ERR_INVALID. d_qkv is [batch*hp*wp][3*heads*dp] fp16 in image
 * order, per token [head][q|k|v][dp] with dp = head_dim rounded up to 16 (16-byte
 * aligned), the single-term layout the forward's QKV GEMM writes (S2S_ATTN=mma and
 * S2S_SPLIT=0 make a forward use that GEMM): q and k L2-normalised, q
 * times exp(min(logit_scale, ln 100)) * log2(e); d_out is [batch*hp*wp][ld_out] fp16, of which columns [0, embed) are
 * written. hp and wp are the padded plane (multiples of the window); odd blocks
 * use the shifted window grid. Work is enqueued on `stream` (NULL = the handle's
 * stream) without synchronising. The first call on each device looks up the
 * array's device address, so make it before any stream capture on that device.
 * Each call rewrites the table before reading it (nothing has to start at zero);
 * overlapping calls on one device race on the table. */
#define S2S_NOALLOC_MAX_TOKENS 1048576
int s2s_window_attention_noalloc(s2s_handle* h, int stage, int block, int batch, int hp, int wp,
                                 const void* d_qkv, void* d_out, int ld_out, void* stream);

/* ---- The image path either side of the forward (src/main.rs:205-224, 365-378:
 * image::load_rgb -> Pre::adjust -> forward -> Image::to_rgb8 -> image::save_rgb).
 * Handle-less calls report errors through s2s_last_error(NULL). */

/* image::load_rgb's header checks (src/image.rs:49-65): width, height, samples per
 * pixel (1 grey, 2 grey+alpha, 3 RGB, 4 RGBA) and bit depth (8 or 16). Indexed
 * colour fails with "unsupported png colour type Indexed", depths below 8 with
 * "unsupported png bit depth One|Two|Four" (S2S_ERR_INVALID). */
int s2s_png_header(const void* png, size_t bytes, int* width, int* height, int* channels,
                   int* bit_depth);

/* Inflate, unfilter and de-interlace (Adam7) into interleaved samples, 16-bit
 * samples big-endian: the buffer the png crate's next_frame fills
 * (src/image.rs:50-52). `capacity` must hold width*height*channels*bit_depth/8. */
int s2s_png_decode(const void* png, size_t bytes, void* samples, size_t capacity);

/* image::save_rgb (src/image.rs:98-114): an 8-bit RGB, non-interlaced PNG of
 * interleaved `rgb` [height][width][3]. Rows are filtered per row (the filter with
 * the least sum of |signed byte|); the zlib stream is deflated at `level` (-1..9,
 * -1 = zlib's default) on `threads` host threads (0 = all cores), each segment
 * primed with the 32 KiB before it. The file is malloc'd into *png (release it
 * with s2s_free); the pixels it decodes to are `rgb` exactly. */
int s2s_png_encode_rgb8(int width, int height, const uint8_t* rgb, int level, int threads,
                        uint8_t** png, size_t* bytes);

/* The same around rows already filtered (s2s_forward_image with png_rows): per row
 * one filter-type byte (0-4) and 3*width filtered bytes. */
int s2s_png_encode_rows(int width, int height, const uint8_t* rows, int level, int threads,
                        uint8_t** png, size_t* bytes);

void s2s_free(void* p);

/* load_rgb's sample scaling (src/image.rs:62-75) fused with Pre::adjust
 * (src/backend.rs:76-86) on the device: `d_samples` [batch][h][w][channels] (8-bit,
 * or 16-bit big-endian) -> `d_chw` [batch][3][h][w] fp32, (s * (1/255 or 1/65535) -
 * mean) * img_range, each operation rounded separately as the host does. */
int s2s_adjust_device(const s2s_handle* h, int batch, int height, int width, const void* d_samples,
                      int channels, int bit_depth, float* d_chw, void* stream);

/* Image::to_rgb8 (src/image.rs:28-39) on the device: [batch][3][h][w] fp32 ->
 * [batch][h][w][3] bytes (clamp to [0,1], * 255, floor(+0.5); NaN -> 255). With
 * `png_rows` non-zero the output is PNG scanlines instead, [batch][h][1 + 3w]: per
 * row the chosen filter type and the filtered bytes, for s2s_png_encode_rows. */
int s2s_rgb8_device(int batch, int height, int width, const float* d_chw, int png_rows,
                    uint8_t* d_out, void* stream);

/* The image path in one call, host buffers, synchronous: decoded samples in
 * ([batch][h][w][channels], 8 or 16 bit), 8-bit RGB out (to_rgb8 layout
 * [batch][h*s][w*s][3], or PNG scanlines [batch][h*s][1 + 3*w*s] with png_rows).
 * `aux` (may be NULL; pixelshuffle_aux only) receives the aux plane in the same
 * format at [batch][hp][wp] (src/main.rs:395-418). Only bytes cross PCIe. */
int s2s_forward_image(s2s_handle* h, int batch, int height, int width, const void* samples,
                      int channels, int bit_depth, int png_rows, uint8_t* out, uint8_t* aux);

/* gpu::selftest (src/gpu.rs:889-1265; `--cuda-selftest`, src/main.rs:179-192): with the
 * same arguments as s2s_create, build handles on `device` and check the fast paths
 * against their plain forms on a seeded two-image batch of an odd size
 * (2*window+3 x 3*window+5): the batch against each image alone (bitwise), a CUDA-graph
 * replay against the eager forward (bitwise), the head convs from kx patches against
 * nine tap boxes (1e-4) and the fused MLP against two GEMMs (2e-3, the parity
 * tolerance: the two sum in different orders). One line per check
 * ("<name> ok|FAILED max-abs <e> (tolerance <t>)") goes to `report` (NUL-terminated, at
 * most `cap` bytes). Returns S2S_OK, S2S_ERR_SELFTEST, or the error that stopped it. */
int s2s_selftest(const s2s_config* cfg, const s2s_tensor* tensors, int n_tensors, int device,
                 char* report, int cap);

void s2s_destroy(s2s_handle* h);

const char* s2s_version(void);

#ifdef __cplusplus
}
#endif

#endif /* S2S_H */
