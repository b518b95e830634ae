/*
 * ixb200.h - C ABI of the B200 (sm_100a) XINT8 YOLOv8 / W4A8 engine, libixb200.so.
 *
 * Plain C: pointers, sizes and POD descriptors only. Every entry point returns 0 or a
 * negative IXB_ERR_* code and never aborts; ixb_last_error() gives a thread-local message
 * (as the reference's ignite_get_last_error, src/ignite_xdna/c_api/ignite.h:157-160 and
 * ignite.cpp:60-64).
 *
 * Which reference interface each entry point replaces:
 *   ixb_session_create   ignite_load (c_api/ignite.h:66-67) and GraphSession.__init__
 *                        (runtime/graph_session.py:775-853): device buffers and weights are
 *                        placed once; here the graph arrives as a plan instead of a container.
 *   ixb_session_run      ignite_run / ignite_run_async (c_api/ignite.h:81-110) and
 *                        GraphSession.run_yolo_monolithic (runtime/graph_session.py:932-989):
 *                        stage_input + dispatch + read_heads for a whole batch.
 *   ixb_session_wait     ignite_wait (c_api/ignite.h:121-126) and RunHandle.wait
 *                        (runtime/session.py:65-84): a timeout is reported, not fatal.
 *   ixb_session_destroy  ignite_free (c_api/ignite.h:133).
 *   ixb_conv_layer, ixb_pool_layer
 *                        one layer of the graph on device buffers, for per-layer parity
 *                        (the reference checks every layer against run_direct,
 *                        results/aie/graph_engine_yolov8n_phoenix_20260913T2210Z.log:12-98).
 *   ixb_i8gemm_srs       int8 x int8 -> int32 GEMM (kernels/int8_matmul_sweep) with the pow2
 *                        SRS epilogue of compiler/engine_emulator.py:149-162 in the int8 domain.
 *   ixb_w4a8_prepare / ixb_w4a8_gemm / ixb_w4a8_gemv
 *                        int8 x packed int4 -> int32 (kernels/w4a8_probe/w4a8_kernels.cc:288-305,
 *                        mm_i8i4_native; operand packing w4a8_probe.py:197-201) plus a
 *                        group-aligned pow2 SRS epilogue.
 */
#ifndef IXB200_H
#define IXB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IXB_OK 0
#define IXB_ERR_INVALID -1    /* bad argument or descriptor */
#define IXB_ERR_CUDA -2       /* a CUDA runtime call failed */
#define IXB_ERR_TIMEOUT -3    /* the host wait ran out */
#define IXB_ERR_DEVICE -4     /* a kernel's bounded wait gave up (device error flag set) */
#define IXB_ERR_UNSUPPORTED -5
#define IXB_ERR_CAPACITY -6   /* more detections survive NMS than the session's capacity */

#define IXB_MAX_SEGS 4
#define IXB_API_VERSION 9

/* Conv A-operand modes. */
#define IXB_MODE_WINDOW 0   /* stride 1, same-resolution inputs: one bulk-copied pixel window per chunk */
#define IXB_MODE_GATHER 1   /* 1x1 conv over a concat with an up2 view: per-pixel cp.async gathers */
#define IXB_MODE_STEM 2     /* 3x3 stride-2 conv over the image tensor (TMA im2col over pixel pairs) */
#define IXB_MODE_IM2COL 3   /* 3x3 stride-2 conv: TMA im2col loads per (tap, chunk) */

/* ixb_session_run flags */
#define IXB_IN_DEVICE 1     /* images is a device pointer; NULL: the images already sit in the staging buffer */
#define IXB_OUT_DEVICE 2    /* egress is a device pointer; NULL: leave the heads in the session's egress buffer */
#define IXB_ASYNC 4         /* return after enqueueing; ixb_session_wait completes the call. Runs
                               stack: a run while one is pending queues behind it on the session's
                               stream, and the wait completes them all (the time is the last run's) */
#define IXB_NO_GRAPH 8      /* launch layer by layer instead of replaying the captured graph */
#define IXB_IN_STORE 16     /* the stem's input already holds the images (ixb_session_letterbox): no ingress */

/* One stored activation tensor, or a channel range of it. Activations are int8 (t = q - 128)
 * stored as one plane per 16-channel chunk: plane c holds [batch][H+2][W+2] pixels of 16 bytes
 * (channels 16c .. 16c+15) with a zero one-pixel halo ring around every image and `guard` zero
 * pixels before and after the plane; IM2COL inputs need plane_stride to be a whole number of
 * images. The image tensor the stem reads is a single guard-free plane of 8-byte pixels
 * (3 channels + 5 zero) [batch][H+2][W+4]: one halo column on the left, three on the right. */
typedef struct ixb_segment {
  uint64_t offset;       /* arena byte offset of padded pixel 0 of image 0 in the tensor's chunk plane 0 */
  uint64_t plane_stride; /* bytes from one chunk plane to the next */
  int32_t chunk_offset;  /* first chunk plane of the view */
  int32_t channels;      /* channels of the view: multiple of 16 (3 for the image tensor) */
  int32_t height;        /* stored height (unpadded) */
  int32_t width;         /* stored width (unpadded) */
  int32_t up2;           /* 1: read as its nearest-2x upsampling */
  int32_t guard;         /* zero pixels before and after every plane: at least (W + 3) (one padded
                            row and pixel) for a 3x3 WINDOW input; a WINDOW conv's tiles are sized so
                            their window copies stay inside it, and guards of 2048 + 2 (W + 3) + 64
                            (what ignite_xdna_b200.plan uses) allow the largest, 2048-row tiles */
} ixb_segment;

/* ixb_conv_desc.out2_kind: a second copy of a conv's output, in the layout its consumer reads. */
#define IXB_OUT2_NONE 0
#define IXB_OUT2_UP2 1      /* nearest-2x upsampled: pixel (y, x) also at (2y + dy, 2x + dx), dy, dx in {0, 1};
                               out2 is (2 out_h) x (2 out_w) x cout */
#define IXB_OUT2_S2D 2      /* space-to-depth for a stride-2 3x3 consumer: pixel (y, x), chunk c also at
                               (y / 2, x / 2), chunk ((y % 2) * 2 + x % 2) * (cout / 16) + c; out2 is
                               (out_h / 2) x (out_w / 2) x 4 cout (out_h, out_w even) */
#define IXB_OUT2_S2D_ONLY 3 /* the space-to-depth copy only (the tensor has no other consumer): `out` unused */

typedef struct ixb_conv_desc {
  int32_t mode;        /* IXB_MODE_* */
  int32_t k, stride;   /* 1 or 3; 1 or 2 */
  int32_t in_h, in_w;  /* logical input size (after any up2) */
  int32_t out_h, out_w;
  int32_t cin, cout;   /* stored channels (whole 16-channel chunks); cout multiple of 16 */
  int32_t n_tile;      /* output channels per CTA (multiple of 16, <= 256, divides cout) */
  int32_t cp;          /* 32-channel pairs of input per K-block */
  int32_t s2d_in;      /* 2: the stem over the image's space-to-depth view (ixb_plan.input_s2d: one
                          chunk holding all four phases; taps as for 1).
                          1: a stride-2 3x3 conv run as a stride-1 2x2 WINDOW conv (k = 2) over the
                          space-to-depth view of its input (IXB_OUT2_S2D): in_h x in_w = out_h x out_w,
                          cin = 4 x the original channels, phase-major; taps at (-1, -1), (-1, 0),
                          (0, -1), (0, 0); only the 9 (phase, tap) pairs of the 3x3 are scheduled */
  int32_t nseg;
  ixb_segment seg[IXB_MAX_SEGS];
  uint64_t w_offset;   /* packed weights: [cout/n_tile][kblocks][block bytes] */
  uint64_t w_bytes;
  uint64_t bias_offset;/* int32[cout]: bias_q << e */
  uint64_t lut_offset; /* int8[256]: activation over t1 + 128 */
  int32_t shift;       /* SRS shift, -31..47 (negative: a saturating left shift; above 16 the
                          epilogue first reduces the accumulator exactly, with a sticky bit) */
  int32_t has_residual;
  ixb_segment residual;
  int32_t res_lsh_main, res_lsh_res, res_shift;
  int32_t out_nchw;    /* 0: write the out view; 1: write int8 NCHW into the egress */
  ixb_segment out;     /* destination view (out_nchw == 0) */
  uint64_t egress_offset;       /* arena offset of this head inside image 0's egress */
  uint64_t egress_image_bytes;  /* egress bytes per image */
  int32_t egress_channels;      /* channels of the head in the egress (<= cout; 0: cout). A head
                                   whose channel count is not a multiple of 16 computes cout =
                                   the next multiple with zero weights and writes only these. */
  int32_t out2_kind;            /* IXB_OUT2_*: the up2 copy lets the top-down path's concat read the
                                   upsampled tensor as a plain tensor with bulk copies instead of
                                   gathering 16-byte rows; the space-to-depth copy turns the stride-2
                                   3x3 convs into stride-1 2x2 convs fed by bulk copies. Not with
                                   out_nchw. */
  int32_t reserved3;
  ixb_segment out2;             /* the second copy's view (out2_kind != IXB_OUT2_NONE) */
} ixb_conv_desc;

typedef struct ixb_pool_desc {  /* SPPF: out_k = pool5^k(in), k = 1..3, pad -128 */
  ixb_segment in;
  ixb_segment out[3];
} ixb_pool_desc;

#define IXB_OP_CONV 0
#define IXB_OP_POOL 1
/* Flag or'ed into a conv op's kind: the conv runs concurrently with the op(s) before it in its
 * branch group (a run of ops joined by this flag, at most IXB_MAX_BRANCHES). No member of a group
 * may read or write what another member writes; session creation checks this on the arena views.
 * The group's members run on separate streams (forked from and joined back into the compute
 * stream, inside the CUDA graph) with the SMs split between them in proportion to their MACs, so
 * small latency-bound convs at 40x40 and 20x20 overlap the large ones instead of each holding
 * the whole GPU for a few microseconds. */
#define IXB_OP_WITH_PREV 0x100
#define IXB_MAX_BRANCHES 8
typedef struct ixb_op { int32_t kind, index; } ixb_op;

#define IXB_MAX_EXTRA_SLOTS 3
typedef struct ixb_plan {
  int32_t api_version;
  int32_t max_batch;
  int32_t img_h, img_w;
  int32_t n_convs, n_pools, n_ops;
  const ixb_conv_desc* convs;
  const ixb_pool_desc* pools;
  const ixb_op* ops;
  uint64_t images_offset;       /* uint8 [max_batch][3][H][W] staging */
  uint64_t input_lut_offset;    /* int8[256]: pixel -> t */
  ixb_segment input;            /* padded 4-byte-pixel image tensor the stem reads */
  uint64_t egress_offset;       /* int8 [max_batch][egress_image_bytes] */
  uint64_t egress_image_bytes;
  uint64_t arena_bytes;
  /* Further staging/egress pairs (same sizes as images_offset / egress_offset) for the
   * ixb_session_submit ring, which is 1 + extra_slots deep; slot 0 is the pair above. */
  int32_t extra_slots;          /* 0 .. IXB_MAX_EXTRA_SLOTS */
  int32_t input_s2d;            /* 1: the stem reads input_s2d_view, the image's space-to-depth view
                                   (16-byte pixels: byte ((y % 2) * 2 + x % 2) * 3 + c holds channel c
                                   of image pixel (y, x), bytes 12..15 zero; (H/2) x (W/2), one chunk,
                                   halo ring and guards like any tensor), which the ingress writes;
                                   `input` then only stages ixb_session_letterbox's output, repacked
                                   into the view before the run */
  uint64_t extra_images_offset[IXB_MAX_EXTRA_SLOTS];
  uint64_t extra_egress_offset[IXB_MAX_EXTRA_SLOTS];
  ixb_segment input_s2d_view;
} ixb_plan;

typedef struct ixb_session ixb_session;

const char* ixb_last_error(void);
int ixb_version(void);

/* Validates every descriptor against the arena (no access outside it) and takes the
 * arena pointer (device memory of arena_bytes, zero-initialised halos, weights in place).
 * arena == NULL: the session allocates and zeroes its own arena. */
int ixb_session_create(const ixb_plan* plan, int device, void* arena, uint64_t arena_bytes, ixb_session** out);
int ixb_session_destroy(ixb_session* s);
void* ixb_session_arena(ixb_session* s);
void* ixb_session_stream(ixb_session* s);    /* the cudaStream_t every launch goes to */
/* Runs the whole network on `batch` images: uint8 [batch][3][H][W] pixels (host memory, or
 * device memory with IXB_IN_DEVICE) -> int8 heads [batch][egress_image_bytes] (host memory,
 * or device memory with IXB_OUT_DEVICE). Copies are issued on the session stream. */
int ixb_session_run(ixb_session* s, const uint8_t* images, int batch, int8_t* egress, int flags);
int ixb_session_wait(ixb_session* s, int timeout_ms);
/* Pipelined asynchronous run, the reference's ignite_run_async / ignite_wait (c_api/ignite.h:102-124):
 * the images are copied in on one copy stream, the network runs on the compute stream, the heads
 * are copied out on another copy stream, all ordered by events. Submitted runs rotate through the
 * plan's 1 + extra_slots staging/egress pairs, so with three slots one run's H2D copy, another's
 * compute and a third's D2H copy proceed together. images / egress are host pointers (pinned, for
 * the copies to overlap) or device pointers; both must stay valid until the ticket completes.
 * Tickets count up from 1; ticket t uses slot (t - 1) % depth, and a submit whose slot is still
 * held by ticket t - depth first waits for it (60 s at most). ixb_session_run is refused while
 * submitted runs are in flight. ixb_session_wait_ticket returns 0 at once for a ticket already
 * collected, and IXB_ERR_TIMEOUT if the run has not finished within timeout_ms. */
int ixb_session_submit(ixb_session* s, const uint8_t* images, int batch, int8_t* egress, uint64_t* ticket);
int ixb_session_wait_ticket(ixb_session* s, uint64_t ticket, int timeout_ms);
/* The compute stream and the two copy streams (cudaStream_t) of a session. */
int ixb_session_streams(ixb_session* s, void** compute, void** h2d, void** d2h);
/* Device milliseconds of the last completed run (CUDA events around the graph launch). */
int ixb_session_last_ms(ixb_session* s, float* ms);
/* Number of kernels one run of `batch` images launches. */
int ixb_session_launches(ixb_session* s, int batch);
/* Runs the network `iters` times layer by layer with an event pair around each launch;
 * writes the mean milliseconds of op i to ms[i] (n_ops entries). */
int ixb_session_profile(ixb_session* s, int batch, int iters, float* ms);
/* Device timeline of one run as it executes in the graph (programmatic dependent launches and
 * branch groups included): runs a copy of the run's graph whose conv launches mark the global
 * timer, `iters` times, and writes for op i of the last run ns[3i..3i+2] = {earliest CTA start,
 * earliest time its inputs were ready (past the wait for the previous kernel), latest CTA end}
 * in globaltimer nanoseconds (n_ops * 3 entries; 0 for pool ops, which do not mark). */
int ixb_session_trace(ixb_session* s, int batch, int iters, uint64_t* ns);

/* One layer on caller-owned device memory: arena is the base every offset refers to. */
int ixb_conv_layer(const ixb_conv_desc* d, void* arena, uint64_t arena_bytes, int batch, void* stream);
int ixb_pool_layer(const ixb_pool_desc* d, void* arena, uint64_t arena_bytes, int batch, void* stream);
/* ixb_conv_layer with per-CTA role counters: stats (device memory, stats_words uint64) receives
 * 16 words per CTA (grid.x * grid.y CTAs, see ixb_conv_launch_info): clock64 cycles the epilogue,
 * MMA and producer roles spent waiting and working, the CTA lifetime and its tile count. */
int ixb_conv_layer_stats(const ixb_conv_desc* d, void* arena, uint64_t arena_bytes, int batch, void* stream,
                         uint64_t* stats, int64_t stats_words);
/* The K schedule of a conv descriptor (shape fields only: mode, k, n_tile, cp, segment channels).
 * kb_out: 8 int32 per K-block {first chunk, chunks, first tap, taps, first MMA, MMAs, weight offset,
 * weight bytes}: A slot s holds chunk (first chunk + s / taps) at tap (first tap + s % taps).
 * ops_out: 6 int32 per MMA {slot, chunk, tap, slot, chunk, tap} of its two 32-byte K-halves; for
 * WINDOW the tap of a half is its window shift; a second half with chunk -1 multiplies zero
 * weights. Returns the number of K-blocks. The packed weights of one n-tile are the MMAs'
 * [n_tile][32] K-slices in this order. */
int ixb_conv_schedule(const ixb_conv_desc* d, int32_t* kb_out, int max_kb, int32_t* ops_out, int max_ops);
/* The launch a conv descriptor gets for `batch` images (host-side decision, no GPU needed):
 * info = {blocks of 128 pixels per tile, tile rows, tiles, pipeline stages, weights resident,
 *         grid.x, grid.y, shared bytes, TMEM columns, K-blocks, A rows per stage, pairs per K-block}. */
int ixb_conv_launch_info(const ixb_conv_desc* d, uint64_t arena_bytes, int batch, int32_t* info, int n);
int ixb_quantize_images(const uint8_t* images, const int8_t* lut, int batch, int h, int w,
                        int8_t* padded_nhwc4, void* stream);

/* int8 GEMM + pow2 SRS (the int8 GEMM of kernels/int8_matmul_sweep with the SRS rule of
 * engine_emulator.py:149-162): out[m][n] = clamp(rne((sum_k a[m][k] * b[n][k] + bias[n]) >> shift),
 * -128, 127), round half to even. a: int8 [M][K] row-major; b: int8 [N][K], i.e. B of C = A.B stored
 * K-major (pass B.T contiguous); bias int32 [N]; out int8 [M][N]. Device pointers, 16-byte aligned;
 * M >= 1, N and K multiples of 16 (pad K with zeros), K <= 65536, shift in [0, 23]. Enqueued on
 * `stream` (a cudaStream_t, NULL for the default stream); returns before the GEMM finishes. */
int ixb_i8gemm_srs(const int8_t* a, const int8_t* b, const int32_t* bias, int8_t* out,
                   int M, int N, int K, int shift, void* stream);
/* Same product without the epilogue: int32 out [M][N] (exact). */
int ixb_i8gemm_i32(const int8_t* a, const int8_t* b, int32_t* out, int M, int N, int K, void* stream);
/* The launch plan of an M x N x K GEMM, or of a W4A8 GEMM when w4a8 != 0 (host only, no GPU
 * needed): {BN, MT, M tiles, N tiles, K blocks, stages, grid, shared bytes, TMEM columns,
 * stage bytes}. */
int ixb_gemm_plan_info(int M, int N, int K, int w4a8, int32_t* info, int n);

/* W4A8: int8 activations x int4 weights with per-group pow2 scales (groups of 128 along K).
 * The weights come in the reference's operand format (kernels/w4a8_probe/w4a8_probe.py:197-201,
 * tools/int4_prefill_model.py:154-200): w_kn uint8 [K][N/2], two int4 per byte along N, element
 * 2j in the low nibble, two's complement; gpos int8 [K/128][N] the group positions (scale
 * exponents). With d = max_g gpos[g][n] - gpos[g][n], which must lie in [0, 4]:
 *   acc[m][n] = sum_g (sum_{k in g} a[m][k] * w[k][n]) << d,
 *   out[m][n] = clamp(rne(acc[m][n] >> shift[n]), -128, 127),  shift int32 [N] in [0, 23].
 * (The reference kernels stop at the raw int32 A.B; the group step is this engine's.)
 * ixb_w4a8_prepare turns (w_kn, gpos) into the engine's weight image (ixb_w4a8_image_bytes of
 * device memory) once; it waits for the stream and refuses a column whose group positions span
 * more than 4. N a multiple of 16, K a multiple of 128, at most 65536; device pointers, 16-byte
 * aligned. ixb_w4a8_gemm (prefill, M rows; tcgen05) and ixb_w4a8_gemv (M = 1; split-K warp
 * reduction) are enqueued on `stream`. */
int ixb_w4a8_image_bytes(int K, int N, uint64_t* bytes);
int ixb_w4a8_prepare(const uint8_t* w_kn, const int8_t* gpos, int K, int N, uint8_t* image, void* stream);
int ixb_w4a8_gemm(const int8_t* a, const uint8_t* image, const int32_t* shift, int8_t* out,
                  int M, int N, int K, void* stream);
int ixb_w4a8_gemv(const int8_t* a, const uint8_t* image, const int32_t* shift, int8_t* out,
                  int N, int K, void* stream);
/* The engine's other operand pair, uint8 activations x int4 weights (the reference's
 * kernels/int4_study/u8i4_kernels.cc mm_u8i4_* and tools/int4_prefill_model.py Int4MmulReference):
 * out int32 [M][N] = sum_k a[m][k] * (w[k][n] << d), a uint8 [M][K], the weight image of
 * ixb_w4a8_prepare (equal group positions give d = 0, the plain product), K <= 32768. */
int ixb_u8i4_gemm_i32(const uint8_t* a, const uint8_t* image, int32_t* out, int M, int N, int K, void* stream);

/* YOLOv8 detect decode + NMS on the GPU: the detections of the reference's
 * pipelines/decode_native.c yolo_decode_int8 (:407-540), bit for bit, for `batch` images of int8
 * heads in the engine's egress layout (device memory, image i at egress + i * egress_image_bytes).
 * Per head: the box and class heads' byte offsets inside an image's egress (int8 NCHW, 4 * 16 and
 * num_classes channels over `anchors`), the tables the reference builds with numpy
 * (dfl_exp float [256][256] 16-byte aligned, sigmoid float [256], sigmoid_low int32 [256] or NULL;
 * pipelines/decode_native.py:125-153) and the prune threshold q_threshold; anchor_x / anchor_y /
 * strides float [sum of anchors] (yolo_pipeline.py:191-203). letterbox float [batch][3] holds
 * pad_top, pad_left, scale per image. Writes per image up to `capacity` detections in NMS order:
 * boxes float [batch][capacity][4] (x0, y0, w, h in source pixels), scores float [batch][capacity],
 * classes int32 [batch][capacity], counts int32 [batch] (-3 where more than `capacity` survive,
 * as the reference). All pointers device memory; reg_max must be 16; at most 8400 anchors and
 * 256 classes per image. Enqueued on `stream`. */
typedef struct ixb_decode_head {
  uint64_t box_offset, cls_offset;
  const float* dfl_exp;
  const float* sigmoid;
  const int32_t* sigmoid_low;
  double q_threshold;
  int32_t anchors, anchor_offset;
} ixb_decode_head;
typedef struct ixb_decode_desc {
  ixb_decode_head head[3];
  const float* anchor_x;
  const float* anchor_y;
  const float* strides;
  int32_t reg_max, num_classes;
  float conf, iou;
} ixb_decode_desc;
int ixb_decode_yolo(const ixb_decode_desc* d, const int8_t* egress, int batch, uint64_t egress_image_bytes,
                    const float* letterbox, int32_t capacity, float* boxes, float* scores, int32_t* classes,
                    int32_t* counts, void* stream);
/* ixb_decode_yolo for callers that may not allocate device memory. No counterpart in the
 * reference. Some callers cannot call cudaMalloc: a plugin running inside a host application that
 * owns the CUDA context and its memory pool, or a loop whose timing cannot take cudaMalloc's
 * implicit synchronisation. Same arguments and detections as ixb_decode_yolo (the caller still
 * passes every input and output); it first ranks the score tables and checks the DFL tables, as a
 * session's detection stage does once, into a 2 KB array of device memory that the library holds
 * on every GPU that loads it until the process exits, and allocates nothing. That scratch holds one
 * table set, so no argument can ask for more. The first call on a device looks up the array's
 * device address: make that first call before any stream capture. Every call uses the same array
 * and rewrites it whole before reading it; calls whose work overlaps on the GPU (on other streams
 * or from other host threads) race on it, so serialise them. Enqueued on `stream`. */
int ixb_decode_yolo_noalloc(const ixb_decode_desc* d, const int8_t* egress, int batch, uint64_t egress_image_bytes,
                            const float* letterbox, int32_t capacity, float* boxes, float* scores,
                            int32_t* classes, int32_t* counts, void* stream);

/* Dense detect decode on the GPU: the reference's InferenceSession.decode_yolo_predictions
 * (runtime/session.py:1223-1278), float32 [batch][4 + num_classes][sum of grid^2] (device memory)
 * from `batch` images of int8 heads (device memory, image i at egress + i * egress_image_bytes).
 * Per level: dequantize v = (q - zero_point) * scale, DFL softmax over 16 bins per box side and
 * its expectation, corners (cell - d) * stride and (cell + d) * stride around the grid cell,
 * centre-size xywh, and the class sigmoid. float32 with CUDA's expf: within a few ulp of the
 * reference's numpy float32, not bit for bit. Enqueued on `stream`. */
typedef struct ixb_dense_head {
  uint64_t box_offset, cls_offset;   /* byte offsets of the 64-channel box and the class head in an image's egress */
  float box_scale;
  int32_t box_zero_point;
  float cls_scale;
  int32_t cls_zero_point;
  int32_t grid;                      /* the level's grid is grid x grid anchors */
  float stride;                      /* pixels per grid cell (8, 16, 32) */
} ixb_dense_head;
int ixb_decode_dense(const ixb_dense_head* heads, int32_t num_classes, const int8_t* egress, int batch,
                     uint64_t egress_image_bytes, float* out, void* stream);

/* Detection stage of a session: the reference's ignite_run / ignite_run_async / ignite_wait
 * contract (c_api/ignite.h:80-125, ignite.cpp:640-980): frames or images in, detections out.
 * After the network, the GPU decode + NMS of ixb_decode_yolo runs on the compute stream and only
 * the detections (counts, boxes, scores, classes) travel back to the host, instead of the heads.
 * ixb_session_set_detect configures it once: the decode descriptor (tables and anchors in device
 * memory owned by the caller, valid while the session uses them), the class heads' scales and zero
 * points (for ixb_session_set_thresholds, the reference's ignite_set_thresholds, ignite.h:141) and
 * the capacity per image (1 .. 8400). It also ranks the score tables and checks the DFL tables
 * once, for every later decode of the session: tables whose contents change afterwards need
 * ixb_session_set_detect again (ixb_decode_yolo derives both in every launch). */
typedef struct ixb_detection {     /* the reference's ignite_detection_t (c_api/ignite.h:40-48) */
  float x0, y0, w, h;              /* top-left corner and size in source-image pixels */
  float score;
  int32_t class_id;
  char class_name[32];             /* from ixb_session_set_class_names, else empty */
} ixb_detection;
typedef struct ixb_timings {       /* the reference's ignite_timings_t (c_api/ignite.h:53-58) */
  double preprocess_ms;            /* letterbox + quantize on the GPU (frames runs; 0 for images runs) */
  double gpu_exec_ms;              /* the network (CUDA events around the graph) */
  double postprocess_ms;           /* decode + NMS on the GPU */
  double glass_to_glass_ms;        /* host clock from the submit to the completed wait */
} ixb_timings;
typedef struct ixb_detect_config {
  ixb_decode_desc decode;
  float cls_scale[3];
  int32_t cls_zero_point[3];
  int32_t capacity;
} ixb_detect_config;
int ixb_session_set_detect(ixb_session* s, const ixb_detect_config* cfg);
int ixb_session_set_thresholds(ixb_session* s, float conf, float iou);
int ixb_session_set_class_names(ixb_session* s, const char* const* names, int n);
/* Pipelined detection runs, ticketed like ixb_session_submit (same ring, same slots):
 * submit_detect takes `batch` uint8 [3][H][W] images at the model size (host or device memory)
 * and optional letterbox rows float [batch][3] (pad_top, pad_left, scale; NULL: none);
 * submit_frames takes `batch` BGR uint8 frames of src_w x src_h (row stride src_stride, frame_bytes
 * apart, host or device memory), copies them in, letterboxes and quantizes them on the GPU
 * (ixb_letterbox_frames) and runs the network on them. Both end with decode + NMS on the GPU and
 * one copy of the detections back. ixb_session_detections waits for the ticket and points into
 * the session's pinned host copy of its detections (valid until the slot is reused, depth submits
 * later): counts [batch] (-3 where more than capacity survive), boxes [batch][capacity][4],
 * scores and classes [batch][capacity]. ixb_session_wait_detections is the reference's ignite_wait:
 * it fills up to max_detections entries for one image and returns how many (IXB_ERR_CAPACITY when
 * more than the capacity survived). ixb_run_frame is the reference's ignite_run: one frame,
 * synchronous. ixb_session_last_timings gives the stages of the last completed detection run. */
int ixb_session_submit_detect(ixb_session* s, const uint8_t* images, int batch, const float* letterbox,
                              uint64_t* ticket);
int ixb_session_submit_frames(ixb_session* s, const uint8_t* frames, int batch, int src_w, int src_h, int src_stride,
                              uint64_t frame_bytes, uint64_t* ticket);
int ixb_session_detections(ixb_session* s, uint64_t ticket, int timeout_ms, int32_t* batch, const int32_t** counts,
                           const float** boxes, const float** scores, const int32_t** classes);
int ixb_session_wait_detections(ixb_session* s, uint64_t ticket, int timeout_ms, int image, ixb_detection* out,
                                int max_detections);
int ixb_run_frame(ixb_session* s, const uint8_t* bgr, int width, int height, int stride, ixb_detection* out,
                  int max_detections);
int ixb_session_last_timings(ixb_session* s, ixb_timings* t);

/* Letterbox ingress, the reference's pipelines/preprocess_simd.c fused_preprocess_bgr_to_c8_plane
 * (:331-590; graph_session.py stage_image :866-889) on the GPU, byte for byte: `batch` BGR uint8
 * frames of src_w x src_h (row stride src_stride, frame_bytes apart; device memory) are letterboxed
 * into dst_w x dst_h with the reference's float32 scale and Q11 bilinear weights and quantized
 * through the int8 input table lut (lut[pixel] = the model input's t = q - 128), as 8-byte pixels
 * (bytes 0..2 = R, G, B; 3..7 untouched) at out (pixel (0, 0) of image 0), rows of out_row_pixels
 * pixels, images out_image_bytes apart. letterbox (host float[3]) receives pad_top, pad_left and
 * scale, the values the decode takes. Enqueued on `stream`. */
int ixb_letterbox_frames(const uint8_t* frames, int batch, int src_w, int src_h, int src_stride, uint64_t frame_bytes,
                         const int8_t* lut, int8_t* out, int dst_w, int dst_h, int out_row_pixels,
                         uint64_t out_image_bytes, float* letterbox, void* stream);
/* The same into a session's stem input, on the session stream; run the network afterwards with
 * ixb_session_run(s, NULL, batch, egress, flags | IXB_IN_STORE). */
int ixb_session_letterbox(ixb_session* s, const uint8_t* frames, int batch, int src_w, int src_h, int src_stride,
                          uint64_t frame_bytes, float* letterbox);

/* sizeof of ixb_segment, ixb_conv_desc, ixb_pool_desc, ixb_plan (for binding checks). */
int ixb_abi_sizes(uint64_t* sizes, int n);

/* Device error flag (bounded waits that gave up); reading clears it. */
int ixb_device_error(int* flag);
/* Self-check of the failure path every kernel's waits share (no reference counterpart: the
 * reference counts NPU dispatch timeouts on the host, c_api/ignite.cpp:929-945): one kernel waits
 * on an mbarrier nothing arrives at, gives up after limit_us microseconds (at most 2 s), raises
 * the device flag and returns. Waits for it on `stream` and returns IXB_ERR_DEVICE when the wait
 * gave up as designed (the flag is then clear again and the context usable). */
int ixb_check_wait_timeout(int limit_us, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* IXB200_H */
