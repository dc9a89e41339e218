// decode.cuh -- input byte tables and the one-to-one YOLO decoder as device kernels.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "unoq_cuda.h"

namespace uq {

constexpr uint32_t kMaxTableChannels = 16;
constexpr uint32_t kMaxDetections = 512;   // records per image and first-stage candidates (sort width)
constexpr uint32_t kMaxAnchors = 32768;
constexpr uint32_t kRankCodes = 1024;

// pixels (uint8, `bytes` in all) -> x: x[i] = table[pixels[i] * channels + i % channels]. `bytes` is
// a multiple of `channels` per image, so i % channels is the channel of byte i of any image.
void launch_pixel_table(const uint8_t *pixels, int8_t *x, size_t bytes, const int8_t *table, uint32_t channels,
                        cudaStream_t s);

// Host-checked summary of an installed decoder (the full UgYoloDecode lives in device memory).
struct YoloShape {
    uint32_t levels = 0, classes = 0, anchors = 0, candidates = 0;
    bool vec = false;  // classes % 16 == 0 and every level's logits 16-byte aligned in the image
};

// One CTA per image: first stage keeps the `min(candidates, anchors)` anchors with the largest
// best-class score (ties: lower anchor first), second stage the `k` largest (anchor, class) pairs
// among them (ties: earlier candidate, then lower class), then each pair's score and pixel box.
void launch_yolo_topk(const int8_t *y, size_t image_bytes, uint32_t images, const UgYoloDecode *cfg,
                      const YoloShape &shape, uint32_t k, UgDetectionRecord *records, cudaStream_t s);

}  // namespace uq
