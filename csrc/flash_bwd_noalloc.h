// Allocation-free entry point of the flash-attention backward.
//
// This entry point has no counterpart in the reference; it is an addition of
// this library for callers that cannot allocate device memory.
//
// Who needs it: a host program that owns every byte of device memory through
// its own pool or arena (an inference server, a game engine, a plugin inside a
// framework with a fixed memory budget) cannot let a library call cudaMalloc
// behind its back: the allocation is outside its budget, can fragment its pool,
// and cudaMalloc/cudaFree may synchronise the device in the middle of its work.
// The regular entry point (dmad_b200._C.flash_bwd) takes its work buffer from
// the caller as a torch tensor; this one needs no buffer at all.
//
// How: the backward's only work buffer, rowsum(dO * O) per query row, lives in
// a file-scope `static __device__` array of DMAD_NOALLOC_MAX_ROWS floats
// (4 MiB, held by every GPU that loads the library until the process exits).
// The caller passes inputs and outputs only.
//
// Rules of use
//   * B * H * round_up(Lq, 256) must not exceed DMAD_NOALLOC_MAX_ROWS; larger
//     problems are rejected with DMAD_NOALLOC_ERR_TOO_LARGE and a message on
//     stderr, nothing is launched.
//   * Every call needs the stream's device current (a stream of another device
//     is rejected with DMAD_NOALLOC_ERR_ARGS).  The first call on a device looks
//     up the device address of the static arrays with cudaGetSymbolAddress;
//     make that first call before any stream capture begins.
//   * q, k, v, o, dout, lse2, dq, dk and dv must start on 16-byte boundaries
//     (they are moved with 16-byte accesses); others are rejected with
//     DMAD_NOALLOC_ERR_ARGS before anything is launched.
//   * Every call shares the one array.  Calls that overlap on the GPU (other
//     streams, other host threads) race on it; serialise them.  The array keeps
//     the last call's contents; each call rewrites every element it reads, so
//     nothing has to start at zero.
//   * The kernels' bounded waits report failures in a status word of the same
//     file, cleared at the start of each call; the return value covers argument
//     and launch errors only (the launch is asynchronous on `stream`).  Read the
//     word with dmad_flash_attn_bwd_noalloc_status after a call: non-zero means
//     a wait gave up and dq / dk / dv are not valid.
#pragma once
#include <cstdint>

#define DMAD_NOALLOC_MAX_ROWS (1 << 20)

enum {
  DMAD_NOALLOC_OK = 0,
  DMAD_NOALLOC_ERR_ARGS = 1,
  DMAD_NOALLOC_ERR_TOO_LARGE = 2,
  DMAD_NOALLOC_ERR_CUDA = 3,
};

#ifdef __cplusplus
extern "C" {
#endif

// Gradients dq, dk, dv of O = softmax(Q K^T * scale) V for bf16 [B, L, H, 128]
// tensors (last dim contiguous; strides in elements, multiples of 8).
//   strides: 24 values, (batch, row, head) strides of q, k, v, o, dout, dq, dk, dv in that order.
//   lse2   : [B, H, round_up(Lq, 256)] fp32 log2-domain row LSE written by the forward.
// Returns DMAD_NOALLOC_OK or an error code.
int dmad_flash_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                const float* lse2, void* dq, void* dk, void* dv, int B, int Lq, int Lk, int H,
                                const int64_t* strides, float scale, void* stream);

// Waits for `stream` and stores the status word of the last call in *out: 0 when every bounded wait of
// the kernels completed, otherwise the code of the wait that gave up.  Allocates nothing.  Returns
// DMAD_NOALLOC_OK, or an error code when the stream is not of the current device or a CUDA call failed.
int dmad_flash_attn_bwd_noalloc_status(void* stream, int* out);

#ifdef __cplusplus
}
#endif
