/*
 * wocr: the inference hot path of huppiflupp/wgpu-ocr (ocrs detector + GRU recogniser, PP-OCR
 * N-D graph executor) as hand-written CUDA for B200 (sm_100a), behind a plain C ABI.
 *
 * Every entry point mirrors a public function of the reference crate (paths are inside the
 * reference repository).  The reference is Rust; its functions return Result<T, String>.  Here
 * each call returns a status code (WOCR_OK = 0) and the message of the last failure on the
 * calling thread is available from wocr_last_error().  Nothing panics or aborts across the ABI.
 *
 * Threading: one wocr_ctx is used by one host thread at a time (the reference's Gpu is not Sync,
 * src/gpu.rs:835-839).  Different contexts, on the same or different GPUs, run concurrently.
 * Ownership: all host buffers are the caller's; weights are copied in at create time, so the
 * caller may free its model description right after a *_create call returns.
 */
#ifndef WOCR_H
#define WOCR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------------------- */
enum {
    WOCR_OK = 0,
    WOCR_ERR_INVALID = 1,     /* bad argument (null pointer, size out of range)            */
    WOCR_ERR_UNSUPPORTED = 2, /* op or attribute the executor does not implement, as the
                                 reference's "unsupported op" errors, src/gpu.rs:1137-1226,
                                 src/nd.rs:1165                                             */
    WOCR_ERR_SHAPE = 3,       /* shapes that do not fit (src/gpu.rs:1322, src/nd.rs:1287)  */
    WOCR_ERR_OOM = 4,         /* device or pinned host allocation failed                   */
    WOCR_ERR_CUDA = 5,        /* a CUDA runtime error                                      */
    WOCR_ERR_TIMEOUT = 6,     /* a bounded wait gave up                                    */
    WOCR_ERR_MISSING = 7,     /* a value or weight the graph names does not exist          */
    WOCR_ERR_CAPACITY = 8     /* an output buffer given by the caller is too small         */
};

/* The message of the last failing call on this thread ("" if none). */
const char *wocr_last_error(void);

/* ---- model description: the loaded ONNX graph --------------------------------------------
 * Mirrors `Onnx` (src/onnx.rs:44-56, filled by Onnx::load src/onnx.rs:88-123): the node list
 * in graph order, float initializers, int64 constants, the graph input and output names.
 * `Constant` nodes are expected already turned into initializers, as Onnx::load does.      */
enum { WOCR_ATTR_INT = 1, WOCR_ATTR_FLOAT = 2, WOCR_ATTR_STRING = 3, WOCR_ATTR_INTS = 4, WOCR_ATTR_FLOATS = 5 };

typedef struct {
    const char *name;
    int32_t kind;         /* WOCR_ATTR_*                                                  */
    int64_t i;            /* WOCR_ATTR_INT                                                */
    float f;              /* WOCR_ATTR_FLOAT                                              */
    const char *s;        /* WOCR_ATTR_STRING                                             */
    const int64_t *ints;  /* WOCR_ATTR_INTS, `count` values                               */
    const float *floats;  /* WOCR_ATTR_FLOATS, `count` values                             */
    int64_t count;
} wocr_attr;

typedef struct {
    const char *op;                   /* ONNX op_type                                     */
    const char *const *inputs;        /* value names ("" for an omitted optional input)    */
    int32_t n_inputs;
    const char *const *outputs;
    int32_t n_outputs;
    const wocr_attr *attrs;
    int32_t n_attrs;
} wocr_node;

/* dtype: 1 = float32, 7 = int64 (ONNX TensorProto codes, src/onnx.rs:58-59). */
typedef struct {
    const char *name;
    int32_t dtype;
    const int64_t *dims;
    int32_t rank;
    const void *data;                 /* prod(dims) values of `dtype`                      */
} wocr_initializer;

typedef struct {
    const wocr_node *nodes;
    int32_t n_nodes;
    const wocr_initializer *inits;
    int32_t n_inits;
    const char *input;                /* first non-initializer graph input (onnx.rs:119)    */
    const char *output;               /* first graph output (onnx.rs:120)                   */
} wocr_model;

/* ONNX model files (src/onnx.rs:57-123, Onnx::load): the protobuf wire format decoded into a
 * wocr_model with the loader's semantics (float / int64 initializers, Constant nodes folded
 * into them, graph input = first input that is not a float weight, output = first output).
 * The model owns its memory until wocr_model_free.  wocr_model_parse reads a buffer. */
int32_t wocr_model_load(const char *path, wocr_model **out);
int32_t wocr_model_parse(const uint8_t *bytes, int64_t n, wocr_model **out);
void wocr_model_free(wocr_model *m);

/* ---- device context: `Gpu` (src/gpu.rs:825-1056) -------------------------------------- */
typedef struct wocr_ctx wocr_ctx;

/* Gpu::new(lines) src/gpu.rs:850: `lines` = lines per GRU recurrence group (LINES, default 8,
 * src/bin/ocr-bench.rs:135).  `device` = CUDA ordinal. */
int32_t wocr_ctx_create(int32_t device, int32_t lines, wocr_ctx **out);
void wocr_ctx_destroy(wocr_ctx *ctx);
/* Device name and capability, as Gpu::adapter (src/gpu.rs:915). */
int32_t wocr_ctx_describe(wocr_ctx *ctx, char *buf, int32_t cap);
/* The CUDA stream (cudaStream_t) all work of this context runs on, as an opaque pointer. */
void *wocr_ctx_stream(wocr_ctx *ctx);
/* Wait for all queued work (Gpu::submit_wait, src/gpu.rs:1005-1008), bounded by timeout_ms
 * (<= 0: no bound).  WOCR_ERR_TIMEOUT when the bound is reached. */
int32_t wocr_ctx_sync(wocr_ctx *ctx, int32_t timeout_ms);
/* Device bytes held by the context's pool (Gpu::pool_bytes, src/gpu.rs:840-845). */
int64_t wocr_ctx_pool_bytes(wocr_ctx *ctx);
/* Number of kernels this context has launched since creation (instrumentation). */
int64_t wocr_ctx_launches(wocr_ctx *ctx);
/* Per-kernel timing (the reference's OPPROFILE/NDPROFILE timers, src/gpu.rs:1247-1368,
 * src/nd.rs:18-27, but with CUDA events on the context stream instead of a wait after every
 * node).  on != 0 starts recording (clearing earlier records), 0 stops. */
int32_t wocr_ctx_profile(wocr_ctx *ctx, int32_t on);
/* Waits for the recorded launches and writes a JSON array of
 * {"kernel", "launches", "ms", "flops", "bytes"} per kernel name into buf (capacity cap). */
int32_t wocr_ctx_profile_report(wocr_ctx *ctx, char *buf, int32_t cap);
/* The same records launch by launch, in launch order: a JSON array of
 * {"kernel", "ms", "flops", "bytes"}. */
int32_t wocr_ctx_profile_launches(wocr_ctx *ctx, char *buf, int32_t cap);
/* Page-locked host memory for fast copies (the caller's staging buffers). */
int32_t wocr_host_alloc(size_t bytes, void **out);
void wocr_host_free(void *p);

/* ---- ocrs detector: `Detector` (src/gpu.rs:1380-1431) --------------------------------- */
typedef struct wocr_detector wocr_detector;

/* Detector::new (src/gpu.rs:1384-1387): the whole model lowered by Graph::build
 * (src/gpu.rs:1104-1240). */
int32_t wocr_detector_create(wocr_ctx *ctx, const wocr_model *model, wocr_detector **out);
void wocr_detector_destroy(wocr_detector *det);

/* Detector::detect_page (src/gpu.rs:1393-1422): packed RGB bytes of a w x h page in, the
 * thresholded bit mask out: h rows of ceil(w / 32) words, bit b of word wx = pixel 32 wx + b. */
int32_t wocr_detect_page(wocr_detector *det, const uint8_t *rgb, int32_t w, int32_t h, float threshold,
                         uint32_t *mask_out);

/* Detector::detect (src/gpu.rs:1425-1430): the model output of a [1, 1, h, w] input, copied to
 * prob_out (capacity `cap` floats; nullable to query the size), its height and width to
 * out_h / out_w. */
int32_t wocr_detect(wocr_detector *det, const float *input, int32_t h, int32_t w, float *prob_out, int64_t cap,
                    int32_t *out_h, int32_t *out_w);

/* Several pages of one size in one pass (the model runs with batch n): `rgb` holds n pages
 * back to back, `mask_out` n masks back to back.  B200 batching of detect_page. */
int32_t wocr_detect_pages(wocr_detector *det, const uint8_t *rgb, int32_t n, int32_t w, int32_t h,
                          float threshold, uint32_t *mask_out);

/* The same on device memory, queued on the context stream without waiting: `d_rgb` and
 * `d_mask_out` are device pointers. */
int32_t wocr_detect_pages_device(wocr_detector *det, const uint8_t *d_rgb, int32_t n, int32_t w,
                                 int32_t h, float threshold, uint32_t *d_mask_out);

/* ---- ocrs recogniser: `Recognizer` (src/gpu.rs:1433-1603) ----------------------------- */
typedef struct wocr_recognizer wocr_recognizer;

/* Recognizer::new (src/gpu.rs:1452-1506): trunk up to the AveragePool, two bidirectional GRU
 * layers (hidden 256, linear_before_reset = 1), MatMul + bias Add output layer. */
int32_t wocr_recognizer_create(wocr_ctx *ctx, const wocr_model *model, int32_t lines, wocr_recognizer **out);
void wocr_recognizer_destroy(wocr_recognizer *rec);

/* Output dimensions of a wocr_recognize call on these batches (without running it). */
int32_t wocr_recognizer_dims(wocr_recognizer *rec, const int32_t *batch_n, const int32_t *batch_w,
                             int32_t n_batches, int32_t *tmax, int32_t *ntot, int32_t *classes);

/* Recognizer::recognize (src/gpu.rs:1510-1602).  Batch b is batch_n[b] line images of
 * 1 x 64 x batch_w[b] floats at batches[b].  Outputs, each nullable:
 *   logits [tmax][ntot][classes] (rows t >= lens[line] are unspecified, as in the reference),
 *   lens   [ntot] (each line's sequence length = its batch's trunk width),
 *   best   [tmax][ntot] arg-max class per step (ties -> the last index, as Rust's max_by),
 * and tmax.  `logits_cap` = capacity of `logits` in floats. */
int32_t wocr_recognize(wocr_recognizer *rec, const float *const *batches, const int32_t *batch_n,
                       const int32_t *batch_w, int32_t n_batches, float *logits, int64_t logits_cap,
                       int32_t *lens, uint32_t *best, int32_t *tmax_out);

/* ---- N-D graph executor: `NdGraph` (src/nd.rs:428-1394) -------------------------------- */
/* The inputs of wocr_ndgraph_run, wocr_ndgraph_run_argmax and wocr_ppdet_page (x, rgb) may be
 * in host or in device memory: they are copied by unified addressing. */
typedef struct wocr_ndgraph wocr_ndgraph;

/* NdGraph::new (src/nd.rs:505-817), with the same load-time fusions. */
int32_t wocr_ndgraph_create(wocr_ctx *ctx, const wocr_model *model, int32_t stop_before_softmax,
                            wocr_ndgraph **out);
void wocr_ndgraph_destroy(wocr_ndgraph *g);

/* NdGraph::run (src/nd.rs:834-1195) on a host tensor; the output is copied to `out`
 * (capacity `out_cap` floats), its shape to out_shape[0..*out_rank) (capacity 6). */
int32_t wocr_ndgraph_run(wocr_ndgraph *g, const float *x, const int64_t *shape, int32_t rank, float *out,
                         int64_t out_cap, int64_t *out_shape, int32_t *out_rank);

/* NdGraph::run + NdGraph::argmax (src/nd.rs:1383-1393): the arg-max over the last axis of the
 * output per row (ties -> the lowest index).  Optionally (nullable) the row maximum and
 * log-sum-exp, so that the softmax probability of the chosen class is exp(max - lse).
 * rows_out = number of rows; `cap` = capacity of each output array. */
int32_t wocr_ndgraph_run_argmax(wocr_ndgraph *g, const float *x, const int64_t *shape, int32_t rank,
                                uint32_t *best, float *row_max, float *row_lse, int64_t cap,
                                int64_t *rows_out, int64_t *out_shape, int32_t *out_rank);

/* ---- record, then read in one wait --------------------------------------------------------
 * The reference records NdGraph::run / NdGraph::argmax_record (src/nd.rs:1372-1380) into one
 * command encoder and reads every recorded buffer with one Gpu::read_many (src/gpu.rs:1011-1037,
 * used at src/bin/ocr-bench.rs:240-253).  A wocr_batch is that read list: each *_enqueue call
 * queues its work on the context stream (nothing waits) and stages a copy of its results in
 * page-locked memory owned by the batch; wocr_wait waits once for the context stream (bounded by
 * timeout_ms, <= 0: no bound) and only then writes every recorded result to the caller's output
 * buffers.  Output buffers must stay valid until wocr_wait returns; an input in page-locked or
 * device memory must stay unchanged until then (pageable inputs are copied before the enqueue
 * returns).  A wait that times out keeps the reads pending for a later wocr_wait.  A batch belongs
 * to one context and is used by that context's thread. */
typedef struct wocr_batch wocr_batch;
int32_t wocr_batch_create(wocr_ctx *ctx, wocr_batch **out);
void wocr_batch_destroy(wocr_batch *b);
/* Number of enqueue calls recorded since the last wocr_wait. */
int64_t wocr_batch_pending(wocr_batch *b);
/* NdGraph::run recorded: arguments as wocr_ndgraph_run, out written at wocr_wait (the shape
 * outputs at once). */
int32_t wocr_ndgraph_run_enqueue(wocr_ndgraph *g, wocr_batch *b, const float *x, const int64_t *shape, int32_t rank,
                                 float *out, int64_t out_cap, int64_t *out_shape, int32_t *out_rank);
/* NdGraph::run + argmax_record: arguments as wocr_ndgraph_run_argmax, best / row_max / row_lse
 * written at wocr_wait (rows_out and the shape at once). */
int32_t wocr_ndgraph_argmax_enqueue(wocr_ndgraph *g, wocr_batch *b, const float *x, const int64_t *shape,
                                    int32_t rank, uint32_t *best, float *row_max, float *row_lse, int64_t cap,
                                    int64_t *rows_out, int64_t *out_shape, int32_t *out_rank);
/* Gpu::read_many: wait for everything recorded in b and deliver it. */
int32_t wocr_wait(wocr_batch *b, int32_t timeout_ms);

/* No counterpart in the reference.  The arg-max of wocr_ndgraph_run_argmax for callers that
 * cannot let the library allocate device memory (a host program whose own allocator owns the
 * GPU, a process under a device-memory cap, a latency-critical path that avoids cudaMalloc's
 * implicit synchronisation).  The caller passes the device logits d_logits [rows][len] (ordered
 * before this call on the context's stream or by a device synchronisation) and host outputs:
 * best [rows] (ties -> the lowest index), and nullable row_max / row_lse [rows].  Results are
 * staged in a fixed 768 KiB array in the library's device memory, for at most 65,536 rows
 * (more rows: WOCR_ERR_CAPACITY); every GPU that loads the library holds that array until the
 * process exits.  Nothing is allocated: no cudaMalloc, cudaFree or allocating routine.  The
 * first call on a device looks up the array's device address (once per device), so make that
 * first call before any stream capture.  With lazy module loading (CUDA's default) that first
 * lookup may also load the library's device code, the array included: make one warm-up call (or
 * set CUDA_MODULE_LOADING=EAGER) before a memory cap starts to matter.  All calls share the
 * array: calls that overlap on the GPU (several contexts or threads at once) race on it. */
int32_t wocr_argmax_rows_noalloc(wocr_ctx *ctx, const float *d_logits, int64_t rows, int64_t len, uint32_t *best,
                                 float *row_max, float *row_lse);

/* NdGraph::det_input (src/nd.rs:1353-1369): the PP-OCR detection input of an RGB page,
 * [1, 3, oh, ow] planar floats, sized as ppdet::det_input (src/ppdet.rs:29-33). */
int32_t wocr_det_input(wocr_ctx *ctx, const uint8_t *rgb, int32_t w, int32_t h, int32_t max_side, float *out,
                       int64_t out_cap, int32_t *ow, int32_t *oh, float *to_page);

/* The PP-OCR detection pass of the reference's GPU thread (src/bin/ocr-bench.rs:186-200):
 * det_input + NdGraph::run on the page, probability map [oh][ow] read back. */
int32_t wocr_ppdet_page(wocr_ndgraph *g, const uint8_t *rgb, int32_t w, int32_t h, int32_t max_side,
                        float *prob, int64_t prob_cap, int32_t *ow, int32_t *oh, float *to_page);

/* DB post-processing on the device (src/ppdet.rs:63-92), on the probability map of the last
 * wocr_ppdet_page call of the handle (which may then pass prob = NULL):
 *   wocr_ppdet_mask:   the map thresholded (p > thresh, as `boxes` builds its mask) into
 *                      [oh][ceil(ow / 32)] words, bit b of word j = pixel 32 j + b;
 *   wocr_ppdet_scores: `score` of each box rects[6 k .. 6 k + 5] = center x, center y, up axis x,
 *                      up axis y, width, height (map coordinates): the mean probability of the
 *                      pixels inside it, summed in the reference's order (bit-exact f32).
 * wocr_ppdet_boxes below runs the whole of `boxes`, contours included, on the device. */
int32_t wocr_ppdet_mask(wocr_ndgraph *g, float thresh, uint32_t *mask, int64_t cap, int32_t *ow, int32_t *oh);
int32_t wocr_ppdet_scores(wocr_ndgraph *g, const float *rects, int32_t n, float *scores);

/* `ppdet::boxes` (src/ppdet.rs:87-132) with the map on the device: the p > thresh mask, its
 * external contours simplified (Douglas-Peucker, epsilon 2) and their minimum-area rectangles
 * (all on the device, as wocr_word_rects), kept when min(width, height) >= min_size and the
 * device `score` >= box_thresh, unclipped by w h unclip_ratio / (2 (w + h)) on every side,
 * dropped when their smaller side is below min_size + 2, scaled to the page (centre by to_page,
 * sides by the factors' mean) and put in reading order (top edge; boxes whose tops are within
 * 10 px ordered by their left edge).  boxes[6 k ..] = center x, center y, up x, up y, width,
 * height; *n = the count (boxes = NULL with cap = 0 only counts; a smaller cap fails with
 * WOCR_ERR_CAPACITY).  ppdet::Db::default(): thresh 0.2, box_thresh 0.45, unclip_ratio 1.4,
 * min_size 3.
 *   wocr_ppdet_boxes: on the map of the handle's last wocr_ppdet_page, with its to_page;
 *   wocr_db_boxes:    on a map [h][w] in host memory, or device memory when prob_on_device. */
int32_t wocr_ppdet_boxes(wocr_ndgraph *g, float thresh, float box_thresh, float unclip_ratio, float min_size,
                         float *boxes, int32_t cap, int32_t *n);
int32_t wocr_db_boxes(wocr_ctx *ctx, const float *prob, int32_t w, int32_t h, int32_t prob_on_device,
                      const float *to_page, float thresh, float box_thresh, float unclip_ratio, float min_size,
                      float *boxes, int32_t cap, int32_t *n);

/* ---- The PP-OCRv6 page pipeline (src/bin/ocr-bench.rs:133-310, 458-585 with PPDET / PPOCR) --
 * One page through detection, DB boxes, line images and recognition, with the page uploaded
 * once and every intermediate (map, bit mask, line batches) kept on the device:
 *   det:   wocr_ppdet_page (max_side), then wocr_ppdet_boxes with db = {thresh, box_thresh,
 *          unclip_ratio, min_size};
 *   lines: each box its own line, grown by relv x its height above and below (the height along
 *          whichever axis is nearer vertical), cut at its bounding rectangle by wocr_pp_lines,
 *          sorted by width into batches of per_batch;
 *   rec:   the recognition graph's arg-max per step of each batch (wocr_ndgraph_run_argmax).
 * Outputs, line by line in reading order: boxes[6 i ..] (before the relv growth), steps[i]
 * (its batch's time steps) and its arg-max classes, concatenated in `best` (cap entries).
 * *n_lines counts the lines; a call with best = NULL and cap = 0 stops after the boxes. */
typedef struct wocr_pp wocr_pp;
int32_t wocr_pp_create(wocr_ctx *ctx, const wocr_model *det, const wocr_model *rec, wocr_pp **out);
void wocr_pp_destroy(wocr_pp *p);
/* Kernels launched so far by all lanes of the pipeline (instrumentation). */
int64_t wocr_pp_launches(wocr_pp *p);
int32_t wocr_pp_page(wocr_pp *p, const uint8_t *rgb, int32_t w, int32_t h, int32_t max_side, const float *db,
                     float relv, int32_t per_batch, float *boxes, int32_t box_cap, int32_t *n_lines,
                     uint32_t *best, int64_t cap, int32_t *steps);

/* Many pages through the same pipeline, as the reference's page loop runs them
 * (src/bin/ocr-bench.rs:458-585 with its GPU thread, 133-310): page k is pages[k] (host or
 * device memory), w[k] x h[k].  The work is spread over `lanes` workers on the pipeline's GPU
 * (each its own stream, graphs and host thread; lane j takes pages j, j + lanes, ...), so one
 * page's detection and recognition overlap another's latency-bound steps.  Each lane holds the
 * line batches of `merge` of its pages (MERGE, src/bin/ocr-bench.rs:162-229) and recognises them
 * together with one wait (wocr_ndgraph_argmax_enqueue + wocr_wait).  Results are those of
 * wocr_pp_page page by page, whatever lanes and merge are: n_lines[k] per page; boxes, steps and
 * best concatenated over the pages in page order (lines in reading order within a page).
 * bytes (nullable) gets {bytes copied host -> device, device -> host}.  A short box_cap or cap
 * fails with WOCR_ERR_CAPACITY after filling n_lines. */
int32_t wocr_pp_pages(wocr_pp *p, const uint8_t *const *pages, const int32_t *w, const int32_t *h, int32_t n,
                      int32_t max_side, const float *db, float relv, int32_t per_batch, int32_t merge, int32_t lanes,
                      float *boxes, int64_t box_cap, int32_t *n_lines, uint32_t *best, int64_t cap, int32_t *steps,
                      int64_t *bytes);

/* Word rectangles of binary page masks: `word_rects` (src/bin/ocr-bench.rs:38-60), i.e. the
 * external contours (find_contours, External), each simplified (Douglas-Peucker, epsilon 2), its
 * minimum-area rectangle resized to width + 2 (expand + expand_x) x height + 2 expand and kept
 * when its area >= min_area (the reference: expand 3, expand_x 0, min_area 100).  `mask`: n
 * pages of h rows x ceil(w / 32) words (bit b of word j = pixel 32 j + b, the layout of
 * wocr_detect_pages), in host memory, or in device memory when mask_on_device != 0.  counts[n]
 * gets each page's rectangle count; rects gets [cx, cy, up_x, up_y, width, height] per
 * rectangle, page after page, each page's in the raster order of its contours' start pixels.
 * rects = NULL with cap = 0 only counts; a cap below the total fails with WOCR_ERR_CAPACITY
 * after filling counts. */
int32_t wocr_word_rects(wocr_ctx *ctx, const uint32_t *mask, int32_t n, int32_t w, int32_t h,
                        int32_t mask_on_device, float expand, float expand_x, float min_area, float *rects,
                        int64_t cap, int32_t *counts);

/* ---- The ocrs page pipeline (src/bin/ocr-bench.rs:458-585 without DET / REC) --------------
 * Text lines from word rectangles: ocrs' find_text_lines (ocrs =0.13.1, called at
 * src/bin/ocr-bench.rs:516; not vendored, restated from its documented behaviour: words ordered
 * by their bounding left edge, each line grown to the right by the nearest word that starts no
 * more than 5 px left of its last word's right edge and overlaps it vertically by 5 px or more;
 * lines by the top of their first word).  words [n][6] = [cx, cy, up_x, up_y, width, height];
 * order[n] gets the word indices line by line (left to right), line_len[*n_lines] the words of
 * each line.  Host only, no device work. */
int32_t wocr_text_lines(const float *words, int32_t n, int32_t *order, int32_t *line_len, int32_t *n_lines);
/* The line padding of src/bin/ocr-bench.rs:534-558 on one line's words (in place): relv x the
 * median word height across the text, relend x it at the line's two ends (ocrs: 0.15, 0.1). */
int32_t wocr_pad_line(float *words, int32_t n, float relv, float relend);
/* ocrs line images from a device-resident RGB page (ocrs' prepare_recognition_input, run on the
 * host by the reference's line_batches, src/bin/ocr-bench.rs:365-408): per line (words
 * concatenated line by line, line_len words each, already padded) its polygon (the words' top
 * edges left to right, then their bottom edges right to left), the polygon's bounding rectangle
 * on the page, pixels outside the polygon -0.5, the others grey, resized to 64 x W
 * (W = clamp(64 width / height, 10, 800)), batched as line_batches batches them: by W rounded up to
 * 50, 20 lines a batch, -0.5 past each line's width.  The batches [n][1][64][width] go one after
 * another to d_out (device, cap floats); slots[i] = the line in batch slot i, widths[i] = its W;
 * batch_n / batch_w per batch; *n_batches and *total (floats) always set, d_out = NULL returns
 * only the layout.  Output arrays may be NULL.  Waits for the device. */
int32_t wocr_ocrs_lines(wocr_ctx *ctx, const uint8_t *d_rgb, int32_t w, int32_t h, const float *words,
                        const int32_t *line_len, int32_t n_lines, float *d_out, int64_t cap, int32_t *slots,
                        int32_t *widths, int32_t *batch_n, int32_t *batch_w, int32_t *n_batches, int64_t *total);

/* The whole ocrs page: Detector::detect_page (threshold), word_rects (expand 3, min area 100),
 * text lines, padding (relv, relend), line images, Recognizer::recognize of the lines of
 * `merge` pages at a time in one pass (MERGE, src/bin/ocr-bench.rs:162-229), arg-max per step
 * (Rust max_by: the last index on ties).  Pages [n] of w x h RGB u8 in host or device memory,
 * spread over `lanes` workers of the pipeline's GPU (each its own stream, detector, recogniser
 * and host thread; lane j takes pages j, j + lanes, ...).  Per page n_lines[k]; per line, pages
 * in order and lines in reading order: line_words (its words), widths (its image width W, for
 * the decode's t * 4 < W rule), steps (its time steps = its batch's trunk width) and its classes
 * concatenated in best; words [Σ line_words][6] the padded words.  Output arrays other than
 * n_lines may be NULL; a capacity below the need fails with WOCR_ERR_CAPACITY after n_lines is
 * filled.  bytes (nullable) = {host -> device, device -> host} bytes of the pages and classes. */
typedef struct wocr_ocrs wocr_ocrs;
int32_t wocr_ocrs_create(wocr_ctx *ctx, const wocr_model *det, const wocr_model *rec, wocr_ocrs **out);
void wocr_ocrs_destroy(wocr_ocrs *p);
int64_t wocr_ocrs_launches(wocr_ocrs *p);
int32_t wocr_ocrs_pages(wocr_ocrs *p, const uint8_t *const *pages, int32_t n, int32_t w, int32_t h, float threshold,
                        float relv, float relend, int32_t merge, int32_t lanes, int32_t *n_lines, int32_t *line_words,
                        int64_t lines_cap, float *words, int64_t words_cap, int32_t *widths, int32_t *steps,
                        uint32_t *best, int64_t cap, int64_t *bytes);

/* Algorithmic work of the last run of a graph handle (detector, recogniser or N-D graph):
 * floating-point operations of its convolutions and matrix products (2 per multiply-add)
 * and the launch count. */
int32_t wocr_last_run_stats(void *handle, int32_t kind, double *flops, int64_t *launches);

/* PP-OCR recognition lines cut from a device-resident RGB page (`d_rgb`, w x h u8) and batched
 * on the device: `ppocr::line_input` (src/ppocr.rs:39-62) for each box rects[4 k .. 4 k + 3] =
 * [left, top, right, bottom] (clamped to the page; resized to height 48 keeping the aspect ratio
 * with the `image` crate's Triangle filter; (v / 255 - 0.5) / 0.5, planar), batched as
 * `pp_batches` (src/bin/ocr-bench.rs:312-345) does: sorted by width, `per_batch` lines a batch,
 * each [n, 3, 48, width], width = the widest line rounded up to 8, zero-padded.  The batches are
 * written one after another to `d_out` (device, `cap` floats).  order[i]: the box of batch slot i;
 * batch_n / batch_w: lines and width of each batch; *n_batches, *total (floats) always set; with
 * d_out NULL only the layout is returned.  Output arrays may be NULL.  Waits for the device. */
int32_t wocr_pp_lines(wocr_ctx *ctx, const uint8_t *d_rgb, int32_t w, int32_t h, const float *rects, int32_t n,
                      int32_t per_batch, float *d_out, int64_t cap, int32_t *order, int32_t *batch_n,
                      int32_t *batch_w, int32_t *n_batches, int64_t *total);

/* Bytes copied host -> device and device -> host by the last call on the handle (same kinds).
 * wocr_detect_pages reports what crossed PCIe for its pages and masks: tall pages go up
 * compacted to the source rows the grey/resize reads.  No reference counterpart (measurement). */
int32_t wocr_last_transfer_bytes(void *handle, int32_t kind, int64_t *h2d, int64_t *d2h);

#ifdef __cplusplus
}
#endif
#endif /* WOCR_H */
