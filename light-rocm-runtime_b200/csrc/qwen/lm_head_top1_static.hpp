// Internal interface of lm_head_top1_static.cu (CUDA runtime code linked into
// liblrrt_qwen.so); the public entry point is lrq_lm_head_top1_static in
// include/lrrt_qwen.h.
#ifndef LRQ_LM_HEAD_TOP1_STATIC_HPP_
#define LRQ_LM_HEAD_TOP1_STATIC_HPP_

#include "lrrt/lrrt.h"
#include "lrrt_qwen.h"

#include <cstdint>
#include <string>

namespace lrq_static {

// Largest grid a call may use: one candidate slot per block (the limit the
// public header documents).
constexpr uint32_t kMaxBlocks = LRQ_STATIC_TOP1_MAX_BLOCKS;

// Runs the kernel on `stream` (a CUstream of the device's primary context),
// waits for it and copies the token and logit to host memory. On failure
// returns the status and fills `error`.
lr_status_t lm_head_top1(uint32_t device, void *stream, const float *lm_head,
                         const float *hidden, uint32_t rows, uint32_t columns,
                         uint32_t blocks, uint32_t *token, float *logit,
                         std::string &error);

} // namespace lrq_static

#endif // LRQ_LM_HEAD_TOP1_STATIC_HPP_
