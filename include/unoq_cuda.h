/*
 * unoq_cuda.h -- C ABI of libunoq_cuda.so, the B200 (sm_100a) backend for unoq-dsp plans.
 *
 * The library is a drop-in for the reference's FastRPC/Hexagon backend. It exports the same
 * symbols with the same argument meaning and error codes, so existing ctypes/FFI callers
 * (unoq_dsp.transport via UNOQ_DSP_LIBRARY, the reference tests via UNOQ_NATIVE_LIBRARY)
 * can load it unchanged. Plans are the reference's UGN1 format (runtime/graph.h:15-38).
 *
 * All buffers named by a plain pointer are HOST memory unless the name says "device".
 * Every call is synchronous unless stated. Error codes:
 *   10-16 header/tensor/matmul validation, 17-19 op validation, 20 work limit,
 *   21 output undefined, 22 bad call, 24 unavailable/poisoned, 25 lifetime overlap
 *   (runtime/graph.c:50-216); 1001 session busy, 1002 allocation, 1003 bad arguments,
 *   1004 transfer, 1005 thread, 1006 timeout (runtime/bridge.c); 2001 CUDA runtime error,
 *   2002 no CUDA device, 2003 device-side wait timed out, 2004 collective failed or timed out.
 */
#ifndef UNOQ_CUDA_H
#define UNOQ_CUDA_H
#include <stddef.h>
#include <stdint.h>
#if defined(__GNUC__)
#define UG_API __attribute__((visibility("default")))
#else
#define UG_API
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* ---- Graph ABI: replaces runtime/graph.h:39-45 (process-global single graph). ---------- */

/* Replaces ug_load (runtime/graph.c:50-262): validate the plan, upload constants, prepare
 * kernels. Any earlier graph is released first. Returns 0 or a 10-25 code. */
UG_API int ug_load(const void *plan, uint32_t bytes);
/* Replaces ug_run (runtime/graph.c:438-448): one image, host buffers, synchronous.
 * A failing run clears the loaded state (reload required), as in the reference. */
UG_API int ug_run(const void *input, uint32_t input_bytes, void *output, uint32_t output_bytes);
/* Allocation-free variant of ug_run (no counterpart in the reference). Same arguments, checks
 * and error codes as ug_run, but the activations live in a fixed 16 MiB device array of this
 * library (the reference's own arena bound, runtime/graph.h:7) instead of memory allocated per
 * batch size, and the ops are launched directly rather than through an instantiated CUDA graph:
 * no cudaMalloc, cudaFree, graph instantiation or other allocating call happens in a call. For
 * callers that may not allocate device memory once running: real-time loops, hosts that forbid
 * allocation after start-up, memory-capped processes. The first call for a loaded graph is its
 * set-up call (host-side layout, the array's device address, first use of the kernels); make it
 * before any stream capture and before allocation is forbidden. A plan whose one-image
 * activations exceed 16 MiB gets 20 and stays loaded. Nothing in the array must start at zero.
 * Overlapping calls on one device would race on the shared array; the graph ABI's lock
 * serialises them within a process. ug_snapshot after this call reads the static array. The
 * ug_profile counters count ug_run calls only, not calls of this variant. */
UG_API int ug_run_static(const void *input, uint32_t input_bytes, void *output, uint32_t output_bytes);
/* Replace ug_input_bytes / ug_output_bytes (runtime/graph.c:263-264); 0 when nothing loaded. */
UG_API uint32_t ug_input_bytes(void);
UG_API uint32_t ug_output_bytes(void);
/* Replaces ug_snapshot (runtime/graph.c:265-268): copy tensor `tensor` of the last image run. */
UG_API int ug_snapshot(uint32_t tensor, void *out, uint32_t bytes);
/* Replaces ug_profile (runtime/graph.c:269-284): command 0 off, 1 reset+on, 2 read.
 * `out` receives (UG_MAX_OP+2) or 130 uint64 counters: [0] runs, [1] total ns,
 * [2+i] nanoseconds spent in op i (CUDA-event timed, profiling runs are not graph-captured). */
UG_API int ug_profile(uint32_t command, void *out, uint32_t bytes);

/* ---- Session ABI: replaces runtime/bridge.c (libuno_backend.so exports). -------------- */

/* Replaces ug_open_mode (runtime/bridge.c:99-125). One active session per process (1001).
 * pipeline 0 = blocking calls; 1 = "mailbox" (bridge.c:161-184): ug_infer then runs one resident
 * CUDA graph per call -- pinned input slot in, the network, pinned output slot out -- and waits
 * for it at most 4 s (1006, as the reference's mailbox response). ug_snapshot_tensor is refused
 * (1003) in mailbox mode, as in the reference; profiling runs take the ordinary path. */
UG_API void *ug_open_mode(const void *plan, uint32_t bytes, int pipeline, int *error);
/* Replaces ug_open (runtime/bridge.c:126). */
UG_API void *ug_open(const void *plan, uint32_t bytes, int *error);
/* Replaces ug_infer (runtime/bridge.c:148-185): one image, host buffers. */
UG_API int ug_infer(void *session, const void *input, uint32_t input_bytes, void *output, uint32_t output_bytes);
/* Replaces ug_close (runtime/bridge.c:70-80); idempotent on NULL. */
UG_API void ug_close(void *session);
/* Replaces ug_snapshot_tensor (runtime/bridge.c:127-130). */
UG_API int ug_snapshot_tensor(void *session, uint32_t tensor, void *out, uint32_t bytes);
/* Replaces ug_profile_control (runtime/bridge.c:134-147). */
UG_API int ug_profile_control(void *session, uint32_t command, void *out, uint32_t bytes);

/* ---- Extensions (no reference counterpart): batching, device selection, timing. ------- */

/* Select the CUDA device used by the next ug_open/ug_load in this process (default 0). */
UG_API int ug_set_device(int device);
/* Run `images` independent images (inputs back to back, outputs back to back), host
 * buffers. Pinned buffers from ug_host_alloc give full-bandwidth copies. The first call
 * for a batch size prepares and captures a CUDA graph for it. From 512 images the batch runs
 * in up to 16 pieces whose host-to-device copy, graph and device-to-host copy overlap on three
 * streams; pieces grow geometrically from a small first one, by the compute/upload time ratio
 * measured on the previous call (UNOQ_PIPE_GROWTH fixes it). */
UG_API int ug_infer_batch(void *session, const void *input, uint32_t images, void *output);
/* Device-resident variant: `device_input`/`device_output` are this session's device
 * buffers from ug_batch_buffers; nothing crosses PCIe. Asynchronous on the session stream. */
UG_API int ug_batch_buffers(void *session, uint32_t images, void **device_input, void **device_output);
UG_API int ug_launch_batch(void *session, uint32_t images);
/* Copy host images into / results out of that device-resident batch (synchronous). */
UG_API int ug_upload_batch(void *session, const void *input, uint32_t images);
UG_API int ug_download_batch(void *session, void *output, uint32_t images);
UG_API int ug_synchronize(void *session);
/* Time `iterations` back-to-back ug_launch_batch(images) on the session stream with CUDA
 * events; writes the elapsed milliseconds. */
UG_API int ug_time_batch(void *session, uint32_t images, uint32_t iterations, float *milliseconds);
/* Milliseconds of the last ug_infer_batch measured by events on the session stream,
 * host-to-device copy, graph and device-to-host copy included. */
UG_API float ug_last_infer_ms(void *session);
/* Pinned host memory for ug_infer_batch buffers. */
UG_API void *ug_host_alloc(size_t bytes);
UG_API void ug_host_free(void *ptr);
/* Host-only loader check with the exact ug_load codes; touches no GPU. */
UG_API int ug_validate_plan(const void *plan, uint32_t bytes);
/* Number of kernel launches one ug_launch_batch issues (graph nodes of this library). */
UG_API int ug_batch_kernel_count(void *session, uint32_t images);
/* Eager profiling of a batch: `iterations` passes with a CUDA event after every plan op;
 * op_ns[i] (count >= number of plan ops) receives the summed nanoseconds of op i and
 * *total_ms the summed pass time. Not graph-captured, so launch gaps are included. */
UG_API int ug_profile_batch(void *session, uint32_t images, uint32_t iterations, uint64_t *op_ns, uint32_t count,
                            float *total_ms);
/* ---- Multi-GPU (extension): one process per GPU, each running a contiguous slice of the
 * global batch; the one collective is the gather of every rank's outputs into rank 0's device
 * memory (NCCL point-to-point over NVLink/NVSwitch, non-blocking mode, every wait bounded). ---- */

/* Rank 0 creates the communicator id (128 bytes) and shares it with the other ranks. */
UG_API int ug_dist_unique_id(void *id, uint32_t bytes);
/* Join the gather (all ranks, same id). Afterwards every ug_launch_batch / ug_time_batch /
 * ug_infer_batch ends with the gather; ug_infer_batch on rank 0 returns the whole gathered batch
 * (world x images outputs, rank-major) in `output`, and returns nothing on the other ranks. */
UG_API int ug_dist_init(void *session, int rank, int world, const void *id, uint32_t bytes);
/* Time `iterations` output gathers alone (no network) of the `images`-image batch on the session
 * stream with CUDA events, after one untimed gather that brings the ranks in step; every rank
 * calls it together. Writes the elapsed milliseconds. */
UG_API int ug_time_gather(void *session, uint32_t images, uint32_t iterations, float *milliseconds);
/* Rank 0's device buffer holding the gathered outputs of `images` per rank (NULL on others). */
UG_API int ug_gather_buffer(void *session, uint32_t images, void **root_device_output);

/* ---- On-device preprocessing and decoding (extension). ------------------------------------
 * The byte table of the image APIs (the reference's modern.py:10-18 profile_lookup and
 * vision.py:20-29 image_lookup: input byte of channel c = table[pixel][c]) and the one-to-one
 * YOLO decoder (modern.py:75-103: distance-to-grid boxes, sigmoid scores, two-stage top-k) run
 * as kernels on the session stream. The host keeps the float-valued pieces that depend only on
 * the model (the tables below, computed with the host decoder's own float32 expressions) and the
 * per-image finish (score threshold, letterbox geometry). */

/* Per-channel input table, `table[256 * channels]` with entry [pixel * channels + c]; NULL (or
 * 0 channels) removes it. While set, every input handed to this session (ug_infer,
 * ug_infer_batch, ug_upload_batch, ug_detect_batch) is uint8 pixels of the input shape, mapped
 * through the table on the device before the network runs. channels: 1..16, dividing the input
 * tensor's bytes. */
UG_API int ug_set_input_table(void *session, const void *table, uint32_t channels);

#define UG_YOLO_MAX_LEVELS 4
typedef struct {
    uint32_t box_offset;    /* byte offset of the level's (h, w, 4) int8 distances in one image's output */
    uint32_t score_offset;  /* byte offset of the level's (h, w, classes) int8 logits */
    uint32_t height, width; /* grid cells */
    float stride;           /* input pixels per cell */
    float distance[256];    /* [q + 128]: dequantised distance, (float(q) - zero_point) * scale in float32 */
    float score[256];       /* [q + 128]: the host decoder's float32 sigmoid of the dequantised logit */
    uint16_t rank[256];     /* [q + 128]: order code of score[] over all levels: equal scores share a code,
                               a larger score has a larger code; codes < 1024 */
} UgYoloLevel;

typedef struct {
    uint32_t levels;        /* 1..UG_YOLO_MAX_LEVELS, anchors numbered level-major, then row-major cells */
    uint32_t classes;       /* 1..4096 */
    uint32_t candidates;    /* anchors kept by the first stage (the reference keeps 300); 1..512 */
    uint32_t reserved;      /* 0 */
    UgYoloLevel level[UG_YOLO_MAX_LEVELS];
} UgYoloDecode;

/* One decoded (anchor, class) pair, in the reference's order: score descending, then first-stage
 * position, then class. Records past the available pairs have anchor = 0xFFFFFFFF. */
typedef struct {
    uint32_t anchor;
    uint32_t class_id;
    float score;
    float box[4];           /* x_min, y_min, x_max, y_max in input pixels: (grid -/+ distance) * stride */
    uint32_t reserved;
} UgDetectionRecord;

/* Install (or, with NULL, remove) the YOLO decoder for this session's plan; the levels' tensors
 * must lie inside the plan's output and the anchors number at most 32768. */
UG_API int ug_set_yolo_decode(void *session, const UgYoloDecode *decode);
/* `images` inputs (host) -> network -> decode; writes images x k records (host), k in 1..512.
 * Same pipelining as ug_infer_batch; multi-rank sessions decode their own shard (no gather). */
UG_API int ug_detect_batch(void *session, const void *input, uint32_t images, uint32_t k, UgDetectionRecord *records);
/* Device-resident variant over the ug_upload_batch context: network + decode on the session
 * stream (asynchronous); ug_detect_buffer gives the device records of (images, k). */
UG_API int ug_launch_detect(void *session, uint32_t images, uint32_t k);
UG_API int ug_detect_buffer(void *session, uint32_t images, uint32_t k, void **device_records);

/* Dense INT8 tensor-core throughput of the selected device, measured: one CTA per SM issues
 * `iterations` rounds of four tcgen05.mma kind::i8 (M 128, N 256, K 32) on shared-memory operands
 * into TMEM; best of three launches, in TOPS (milliseconds of that launch optional). The roofline
 * denominator of the tensor-core convolutions. */
UG_API int ug_measure_int8_peak(uint32_t iterations, float *tops, float *milliseconds);

/* Last CUDA error string seen by the library (empty if none). */
UG_API const char *ug_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
