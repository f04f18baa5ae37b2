/*
 * qppocr_cuda.h — C ABI of libqppocr_cuda.so, the B200 (sm_100a) device
 * backend for qppocr.
 *
 * It fills the reference's CUDA stub (crates/qppocr-gpu/src/cuda.rs:112-230,
 * whose create_session returns "kernels not implemented") behind the
 * backend-agnostic device seam of qppocr-core:
 *   trait DeviceContext  (crates/qppocr-core/src/device.rs:83-101)
 *   trait DeviceSession  (crates/qppocr-core/src/device.rs:125-176)
 *   trait DeferredRun    (crates/qppocr-core/src/device.rs:105-108)
 * A thin Rust FFI crate (qppocr-cuda) binds these symbols and implements the
 * traits.
 *
 * Conventions: every function returns int status (QPC_OK == 0).  On failure,
 * qpc_last_error() returns a thread-local message naming the node, op or CUDA
 * call — the same "no silent fallback" discipline as Error::Graph /
 * Error::Device (crates/qppocr-core/src/error.rs:15-18).  Plain pointers and
 * sizes only; tensors are fp32 row-major (logical NCHW) on the host side.
 * Sessions are safe to use from many threads at once (device.rs:120-125).
 */
#ifndef QPPOCR_CUDA_H
#define QPPOCR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define QPC_OK 0
#define QPC_ERR_INVALID 1 /* bad argument (null pointer, wrong count, ...) */
#define QPC_ERR_GRAPH 2   /* Error::Graph: unsupported op / shape, missing tensor */
#define QPC_ERR_DEVICE 3  /* Error::Device: no device, CUDA failure, kernel fault */
#define QPC_ERR_TIMEOUT 4 /* qpc_complete deadline passed (run still in flight) */
#define QPC_ERR_OOM 5     /* device or pinned-host allocation failed */

/* Message of the last failing call on this thread ("" if none).
 * Replaces the Error::Device / Error::Graph strings (error.rs:15-18). */
const char* qpc_last_error(void);

/* ------------------------------------------------------ device discovery */
/* Number of CUDA devices (0 when the driver is absent is not an error).
 * Replaces enumerate() (crates/qppocr-gpu/src/cuda.rs:63-110). */
int qpc_device_count(int* count);

/* Name, driver version (e.g. 12090) and compute capability of one device.
 * Replaces CudaContext::open + DeviceContext::info (cuda.rs:121-212).
 * Fails with QPC_ERR_DEVICE for an out-of-range index or a device that is
 * not sm_100 (this library carries sm_100a code only). */
int qpc_device_info(int device, char* name, int name_len, int* driver_version, int* cc_major,
                    int* cc_minor);

/* -------------------------------------------------- graph description
 * Mirrors the reference's in-memory ONNX model (crates/qppocr-core/src/
 * onnx/model.rs:13-127) as handed to DeviceContext::create_session: the graph
 * has already been through the load-time passes (BN folded into Conv, Conv
 * carries `act` (0/1 gelu/2 relu) + act_c1..3, bias in inputs[2], residual in
 * inputs[3]; Add(Mul(f, g), r) collapsed to MulAddScale), see
 * crates/qppocr-core/src/onnx/parse.rs:731-747. */
enum qpc_attr_kind {
  QPC_ATTR_FLOAT = 1,  /* Attribute.f      (field 2) */
  QPC_ATTR_INT = 2,    /* Attribute.i      (field 3) */
  QPC_ATTR_STRING = 3, /* Attribute.s      (field 4) */
  QPC_ATTR_FLOATS = 4, /* Attribute.floats (field 7) */
  QPC_ATTR_INTS = 5    /* Attribute.ints   (field 8) */
};

typedef struct {
  const char* name;
  int kind; /* qpc_attr_kind */
  float f;
  int64_t i;
  const char* s;
  const float* floats;
  const int64_t* ints;
  int n; /* length of floats / ints */
} qpc_attr;

typedef struct {
  const char* op_type; /* "Conv", "MatMul", ... (Node.op_type) */
  const char* name;
  const char* const* inputs; /* "" = absent optional input */
  int n_inputs;
  const char* const* outputs;
  int n_outputs;
  const qpc_attr* attrs;
  int n_attrs;
} qpc_node;

typedef struct {
  const qpc_node* nodes; /* topological order (Graph.nodes) */
  int n_nodes;
  const char* const* inputs; /* Graph.inputs */
  int n_inputs;
  const char* const* outputs; /* Graph.outputs */
  int n_outputs;
} qpc_graph;

/* tensor.rs:10-18 DType.  QPC_U8_IMAGE (run inputs only; no counterpart in
 * the reference's DType) is a batch of n x h x w x 3 uint8 RGB images given
 * for an f32 graph input of shape [n, 3, h, w]: the session normalises it on
 * the device exactly as the reference engine prepares the det input,
 * v = u8 * (1/255), (v - 0.5) * (1/0.5), HWC -> CHW (engine.rs:963-982), so
 * a run moves a quarter of the bytes across the host and PCIe. */
/* QPC_F32_DEVICE (run inputs only; no counterpart in the reference) is an
 * f32 tensor already in this device's memory (`data` is a device pointer): the
 * run copies it device-to-device on its own stream, so a caller that prepared
 * the input on the GPU (qpc_op_rec_pack, qpc_op_det_preprocess) hands it over
 * without a host round trip.  The data must be complete before the call (make
 * the producing stream finish first) and stay unchanged until the run
 * completes.  Same plans as QPC_F32. */
/* QPC_U8 (outputs only): a uint8 tensor, the det mask exit's mask.
 * QPC_U8_IMAGE_DEVICE (run inputs only): a QPC_U8_IMAGE batch already in this
 * device's memory (same rules as QPC_F32_DEVICE), e.g. images a pipeline also
 * crops text lines from on the device. */
enum qpc_dtype {
  QPC_F32 = 0,
  QPC_I64 = 1,
  QPC_U8_IMAGE = 2,
  QPC_F32_DEVICE = 3,
  QPC_U8 = 4,
  QPC_U8_IMAGE_DEVICE = 5
};

/* A host tensor (tensor.rs:28-40): initializers and run inputs. */
typedef struct {
  const char* name;
  const int64_t* shape;
  int rank;
  int dtype; /* qpc_dtype */
  const void* data;
} qpc_tensor;

/* ---------------------------------------------------------------- session */
/* ModelRole (device.rs:53-66). */
enum qpc_role { QPC_ROLE_OTHER = 0, QPC_ROLE_DET = 1, QPC_ROLE_REC = 2, QPC_ROLE_CLS = 3 };

/* Math of the tensor-core contractions (QPPOCR_CUDA_MATH). */
enum qpc_math { QPC_MATH_TF32 = 0, QPC_MATH_3XTF32 = 1 };

typedef struct {
  int math;                  /* qpc_math; default TF32 */
  int argmax_exit;           /* rec: emit [B,T,2] (val, idx bits) instead of [B,T,C]
                                (DeviceSession::rec_argmax_pairs, device.rs:159-163);
                                -1 = role default (on for REC) */
  int64_t plan_budget_bytes; /* plan cache byte budget (idle plans evicted oldest first when a
                                new one would exceed it); 0 = default, a quarter of the
                                device's memory (at least 8 GiB) */
  int use_cuda_graph;        /* 1 = one captured CUDA graph per shape (default), 0 = stream launches */
  int det_mask_exit;         /* det (role DET, one [n,1,h,w] output): output 0 becomes the [n,h,w]
                                QPC_U8 mask pred > mask_thresh, 2x2-dilated when mask_dilate
                                (the DB post's first step, geometry.rs:286-296), and output 1 the
                                probability map, kept in device memory (no host copy) for
                                qpc_op_box_score; 0 = off */
  float mask_thresh;         /* DB binarize threshold (PipelineConfig det_db_thresh; default 0.3) */
  int mask_dilate;           /* 1 = 2x2 dilation (use_dilation) */
} qpc_session_options;

typedef struct qpc_session qpc_session;

/* DeviceContext::create_session (device.rs:88-101): the session takes a host
 * copy of the weights and owns them; each is uploaded to the device once, in
 * the layout its kernel wants, when the first run that needs it builds its
 * plan (so a device out-of-memory surfaces at that run as QPC_ERR_OOM).
 * Unsupported ops fail here, naming the node (QPC_ERR_GRAPH).  opts may be
 * NULL (defaults). */
int qpc_session_create(int device, const qpc_graph* graph, const qpc_tensor* weights,
                       int n_weights, int role, const qpc_session_options* opts,
                       qpc_session** out);

/* Capability queries of DeviceSession (device.rs:134-163). */
typedef struct {
  int prefers_host_parallelism; /* prefers_host_parallelism()  :134 (GPU: 0) */
  int bucket_grain;             /* bucket_grain()              :139 (GPU: 64) */
  int batch_grain;              /* batch_grain()               :148 */
  int rec_chunk;                /* rec_chunk()                 :157 */
  int argmax_pairs;             /* rec_argmax_pairs()          :163 */
} qpc_caps;
int qpc_session_caps(const qpc_session* s, qpc_caps* caps);

/* A run in flight or completed (DeferredRun, device.rs:105-108). */
typedef struct qpc_ticket qpc_ticket;

/* DeviceSession::run_deferred (device.rs:164-176): stage the inputs, launch
 * the shape's captured graph and return at once.  Two runs of the same shape
 * may be in flight: the session keeps a separate plan instance per run
 * (inputs/outputs never share buffers). */
int qpc_run_async(qpc_session* s, const qpc_tensor* inputs, int n_inputs, qpc_ticket** ticket);

/* DeferredRun::complete: wait (bounded by timeout_ms; <0 = no bound) for the
 * run, check for device faults.  On QPC_ERR_TIMEOUT the ticket stays valid. */
int qpc_complete(qpc_ticket* ticket, int timeout_ms);

/* Outputs of a completed ticket in graph-output order (DeviceSession::run
 * return value, device.rs:130).  *data stays valid until qpc_ticket_release. */
int qpc_ticket_output_count(const qpc_ticket* ticket, int* count);
int qpc_ticket_output(const qpc_ticket* ticket, int index, const float** data,
                      const int64_t** shape, int* rank);
/* Type and place of output `index` of a completed ticket: *dtype a
 * qpc_dtype (QPC_F32, or QPC_U8 for the det mask), *device_only 1 when the
 * output stays in device memory (qpc_ticket_output then gives data NULL), and
 * *device_data its device address, valid until qpc_ticket_release.  Any
 * pointer may be NULL. */
int qpc_ticket_output_info(const qpc_ticket* ticket, int index, int* dtype, int* device_only,
                           const void** device_data);
/* Copy output `index` of a completed ticket into the caller's buffer `dst`
 * (`count` elements of the output's dtype, its element count) with the library's host copy
 * threads.  This is the copy into the fresh host Tensor that
 * DeviceSession::run returns (device.rs:130); a binding may instead copy
 * from qpc_ticket_output's pointer itself. */
int qpc_ticket_output_copy(const qpc_ticket* ticket, int index, float* dst, int64_t count);

/* Pinned (page-locked) host memory for run inputs (extension; the reference's
 * host tensors are plain Vec<f32>).  A run input whose bytes lie wholly in one
 * such block is copied to the device by DMA straight from it, with no staging
 * copy; the caller keeps it unchanged until the ticket completes.  Outputs are
 * always delivered in pinned memory (qpc_ticket_output). */
int qpc_host_alloc(int64_t bytes, void** ptr);
int qpc_host_free(void* ptr);
int qpc_ticket_release(qpc_ticket* ticket);

/* DeviceSession::run (device.rs:130): run_async + complete(no bound). */
int qpc_run(qpc_session* s, const qpc_tensor* inputs, int n_inputs, qpc_ticket** ticket);

/* Device time (ms, CUDA events on the run's stream) of a completed ticket. */
int qpc_ticket_device_ms(const qpc_ticket* ticket, float* ms);

int qpc_session_destroy(qpc_session* s);

/* ------------------------------------------------------- diagnostics
 * Per-step device timing and kernel-only replay, the counterpart of the
 * reference's QPPOCR_GPU_PROF per-dispatch timestamps
 * (crates/qppocr-gpu/src/vulkan/session.rs:828-835, 2073-2139). */

/* Run the plan for these input shapes `iters` times with CUDA events between
 * steps; *n_steps = number of steps (kernel launches). */
int qpc_session_profile(qpc_session* s, const qpc_tensor* inputs, int n_inputs, int iters,
                        int* n_steps);
/* Step `idx` of the last profile: kernel family, graph node, algorithmic DRAM
 * bytes and flops of one launch, mean device ms. */
int qpc_session_profile_step(const qpc_session* s, int idx, const char** kernel,
                             const char** node, double* bytes, double* flops, float* ms);
/* Stage inputs once, then replay the shape's compute graph `iters` times back
 * to back; *ms_per_replay = device ms per replay (no host copies inside). */
int qpc_session_replay(qpc_session* s, const qpc_tensor* inputs, int n_inputs, int iters,
                       float* ms_per_replay);

/* The session's node list after load-time fusion: op ("Conv", "QpcLinear",
 * "QpcLayerNorm", ...), node name and first output tensor.  Making those
 * outputs graph outputs of a second session changes no fusion, so every
 * fused node can be compared on its own (dump-compare stepping,
 * QPPOCR_GPU_DUMP_CMP, crates/qppocr-gpu/src/vulkan/session.rs:542-600). */
int qpc_session_node_count(const qpc_session* s, int* n);
int qpc_session_node(const qpc_session* s, int idx, const char** op, const char** name,
                     const char** output);

/* ------------------------------------------------ operator entry points
 * Device-pointer entry points for single operators (the qppocr-kernels
 * functions the session composes), for callers that manage device memory
 * themselves and for operator-level parity tests.  All pointers are device
 * pointers, 16-byte aligned; `stream` is a cudaStream_t (NULL = legacy).
 * Activations are NHWC fp32.  act: 0 none, 1 relu, 2 hardswish
 * (x * HardSigmoid(x; alpha, beta)), 3 sigmoid, 4 gelu, 5 hardsigmoid,
 * 6 swish; act_p = {alpha, beta, c1, c2, c3} (NULL = PP-OCR defaults
 * 1/6, 1/2, sqrt2, 1, 0.5). */

/* Depthwise conv, group == C.  Replaces conv2d_res_into's depthwise branch
 * (crates/qppocr-kernels/src/conv.rs:461-505, plane kernel :45-71) and
 * depthwise_nhwc_packed (conv.rs:912-1051).  w_tap_major: [kh*kw][c].
 * pads: {ph, pw, peh, pew}; strides {sh, sw}; residual may be NULL. */
int qpc_op_dwconv_nhwc(const float* x, int n, int h, int w, int c, const float* w_tap_major,
                       int kh, int kw, const int* strides, const int* pads, const float* bias,
                       int act, const float* act_p, const float* residual, float* y,
                       void* stream);

/* Pointwise conv / linear layer on tcgen05 tensor cores:
 * y[M,N] = act(x[M,K] * w[N,K]^T + bias) + residual.  Replaces the 1x1 path
 * of conv2d_res_into (conv.rs:264-460 -> sgemm_res, gemm.rs:53-66, 223-466),
 * conv1x1_nhwc (conv.rs:856-901) and constant-B matmul (shape.rs:568-653).
 * math: qpc_math.  x is rounded to tf32 (nearest) on chip; w should already
 * be tf32-rounded: pass the `hi` part of qpc_op_split_tf32 as w, and for
 * QPC_MATH_3XTF32 its `lo` part as w_lo (ignored for TF32). */
int qpc_op_gemm(const float* x, int64_t m, int k, const float* w, const float* w_lo, int n,
                const float* bias, int act, const float* act_p, const float* residual, float* y,
                int math, void* stream);

/* Fused CTC head with the argmax exit (rec MatMul 120 -> V + bias + Softmax +
 * per-timestep argmax; crates/qppocr-core/src/pipeline/rec.rs:34-120 and
 * crates/qppocr-gpu/shaders/n_exit3_argmax.comp): for each of `rows` rows of
 * x[rows, k], pairs[2r] = softmax probability of the first strict maximum of
 * x * w^T + bias (ties -> lowest class), pairs[2r+1] = its class index as an
 * f32 bit pattern.  w is [n, k] tf32-rounded (and w_lo as for qpc_op_gemm).
 * The logits are never written: a scratch buffer of per-column-tile partials
 * (rows * ceil(n / 128) * 16 bytes) is allocated and freed stream-ordered. */
int qpc_op_ctc_head(const float* x, int64_t rows, int k, const float* w, const float* w_lo, int n,
                    const float* bias, int math, float* pairs, void* stream);

/* qpc_op_ctc_head without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot let a library allocate GPU
 * memory (an engine that owns all device memory in its own pool, or a serving
 * loop that must not call the CUDA allocator once running).  Same arguments
 * and result as qpc_op_ctc_head; the partials live in a fixed array compiled
 * into this library (32 MiB per device, held until process exit).
 * Limit: rows x (column tiles of n) <= 2^21 entries, else QPC_ERR_INVALID;
 * rows * ceil(n / 128) <= 2^21 is sufficient.  All calls on a device share
 * that array: calls whose kernels overlap on the GPU race.  A pipeline wait
 * that runs out is kept (in a fixed word, not allocated) until
 * qpc_kernel_error reads it.  The first call on a device looks up the
 * array's address (cudaGetSymbolAddress); make it before any stream capture. */
int qpc_op_ctc_head_noalloc(const float* x, int64_t rows, int k, const float* w, const float* w_lo,
                            int n, const float* bias, int math, float* pairs, void* stream);

/* Split fp32 device values into tf32 parts hi = rn(v) and lo = rn(v - hi)
 * (round to nearest, ties away): the load-time weight preparation of both
 * math modes. */
int qpc_op_split_tf32(const float* v, int64_t count, float* hi, float* lo, void* stream);

/* ------------------------------------------------ det / rec pre and post
 * Device versions of the host code on either side of the networks, bit-exact
 * with it.  Device pointers; images are n x h x w x 3 uint8 (HWC, as the
 * reference's `Image`), masks n x h x w uint8. */

/* resize_bilinear_img / resize_bilinear_rgb_u8 (crates/qppocr-core/src/
 * pipeline/image.rs:50-117, crates/qppocr-kernels/src/resize.rs:158-210): the
 * det input resize and the rec line resize, n images sh x sw -> dh x dw. */
int qpc_op_resize_bilinear_rgb_u8(const uint8_t* src, int n, int sh, int sw, uint8_t* dst, int dh, int dw,
                                  void* stream);

/* Det input preparation (crates/qppocr-core/src/pipeline/engine.rs:930-982):
 * resize to dh x dw (skipped when the sizes are equal, as there), then
 * v = u8 * (1/255), (v - 0.5) * (1/0.5) into planar n x 3 x dh x dw f32 -
 * the det session's input tensor. */
int qpc_op_det_preprocess(const uint8_t* src, int n, int sh, int sw, float* dst, int dh, int dw, void* stream);

/* Rec line pack (crates/qppocr-core/src/pipeline/crop.rs:153-185 pack_crop
 * into the zeroed batch tensor of engine.rs:1425-1440): n uint8 crops (h[k] x
 * w[k] x 3 at byte offset off[k] of `crops`) -> n x 3 x img_h x img_w f32;
 * line k is resized to rw[k] x img_h (bilinear, as resize_bilinear_img), then
 * v = u8 / 255, (v - 0.5) / 0.5; with pad[k] != 0 it is placed unresized,
 * centred vertically.  Other positions are 0.  All arrays in device memory. */
int qpc_op_rec_pack(const uint8_t* crops, const int64_t* off, const int* h, const int* w, const int* rw,
                    const int* pad, int n, int img_h, int img_w, float* out, void* stream);

/* DB post-processing mask (crates/qppocr-core/src/pipeline/geometry.rs:
 * 286-296 with qppocr-kernels resize.rs:213-245 dilate2x2_max): mask =
 * pred > thresh, then, when `dilate`, the 2x2 dilation (window [y-1, y] x
 * [x-1, x], out-of-bounds samples ignored).  pred: n x h x w probabilities;
 * the mask feeds the host's connected components.  With pred == NULL,
 * mask_in (uint8) is dilated instead. */
int qpc_op_db_mask(const float* pred, const uint8_t* mask_in, uint8_t* mask, int n, int h, int w, float thresh,
                   int dilate, void* stream);

/* box_score_fast (crates/qppocr-core/src/pipeline/geometry.rs:221-269) on
 * the device: for box k, the mean (f64 sum in the reference's order, rounded
 * to f32) of pred over the quadrilateral boxes[8k .. 8k+7] ((x, y) corners in
 * pred's coordinates) of image img[k] by the scan-line even-odd fill; 0 for
 * an empty box.  pred: n x h x w probabilities; boxes, img, scores device
 * arrays.  The DB post's score filter without copying the map to the host. */
int qpc_op_box_score(const float* pred, int h, int w, const float* boxes, const int* img, int n_boxes,
                     float* scores, void* stream);

/* Host helper for qpc_op_crop_text_boxes: the size of crop_text_box's output
 * for each box (crates/qppocr-core/src/pipeline/crop.rs:9-15): cw = max(1,
 * max(|p0 p1|, |p2 p3|) truncated), ch likewise from |p0 p3|, |p1 p2| (f32
 * hypot); rotated[k] = ch / cw >= 1.5 (the crop is then ch wide, cw high).
 * pts: host array [n][4][2]. */
int qpc_crop_size(const float* pts, int n, int* cw, int* ch, int* rotated);

/* crop_text_box (crop.rs:8-127) on the device: box k of image img[k] (n_images
 * images of h x w x 3 uint8, device) -> cw[k] x ch[k] x 3 bytes at out +
 * off[k], the f64 homography solve, f64 inverse mapping and edge-replicated
 * bilinear sampling of the reference, bit for bit; tall crops rotated
 * clockwise.  pts, img, cw, ch, off: device arrays; max_pixels: the largest
 * cw * ch. */
int qpc_op_crop_text_boxes(const uint8_t* images, int n_images, int h, int w, const float* pts, const int* img,
                           const int* cw, const int* ch, const int64_t* off, int n_boxes, int max_pixels,
                           uint8_t* out, void* stream);

/* Line pack on the device (pack_crop, crop.rs:153-185, into the zeroed batch
 * of engine.rs:1425-1440): line k is the view of an h[k] x w[k] window,
 * starting at column x0[k], of a crop whose rows are stride[k] pixels, at
 * byte offset off[k] of crops; flip[k] != 0 rotates the view 180 degrees (a
 * line the classifier flagged, engine.rs:1402-1407; flip may be NULL).  The
 * view is resized to rw[k] x img_h (bilinear, as resize_bilinear_img) and
 * normalised (v/255 - 0.5)/0.5, or with pad[k] != 0 placed unresized and
 * centred vertically, into slot k of out (n x 3 x img_h x img_w f32).  The
 * cls batch is this with cls_view's centred window (crop.rs:193-218) and
 * pad 0; the rec batch with the whole crop.  All arrays on the device. */
int qpc_op_line_pack(const uint8_t* crops, const int64_t* off, const int* stride, const int* x0, const int* h,
                     const int* w, const int* rw, const int* pad, const int* flip, int n, int img_h, int img_w,
                     float* out, void* stream);

/* Device fault / timeout flags raised by kernels with bounded waits on
 * `device` since the last call (0 = none; 1 = a pipeline wait ran out, 2 = a
 * kernel saw an impossible shape), including the faults kept by
 * qpc_op_ctc_head_noalloc; clears them.  Session runs read them after every
 * run and fail with QPC_ERR_DEVICE. */
int qpc_kernel_error(int device, unsigned int* flags);

/* ------------------------------------------------ failure-path self-tests
 * Host-driven checks of the error paths that need no real fault (the
 * reference's failure handling: no silent fallback, bounded device waits,
 * crates/qppocr-core/src/device.rs:88-94, vulkan/session.rs:306-312). */

/* Launch one CTA that waits, with the bounded wait of the pipelined kernels
 * and a limit of limit_us microseconds (1 .. 1e6), on an mbarrier nothing
 * arrives on, and wait for it to return.  path 0 reports into the device's
 * fault word, path 1 into the word of qpc_op_ctc_head_noalloc (as its kernels
 * would after a timed-out wait).  Either way qpc_kernel_error(device) then
 * returns flag 1 and the device stays usable. */
int qpc_selftest_wait_timeout(int device, int path, int limit_us);

/* Make the nth device allocation of the library from now on (1 = the next
 * one; 0 cancels) fail as if the device were out of memory: the call that
 * makes it returns QPC_ERR_OOM and leaves no state behind. */
int qpc_inject_alloc_failure(int nth);

#ifdef __cplusplus
}
#endif

#endif /* QPPOCR_CUDA_H */
