// Host/device interface of the tensor-core GEMM family (tcgen05 + TMA).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "grx/grx_cycles.h"

namespace grx {

// Versioned argument block, passed by value as a __grid_constant__ parameter.
// The kernel refuses to run on a version mismatch (the reference's kernel ABI
// blocks do the same, src/libs/grxblas/hgemm_abi.h:20 and
// src/libs/grxblas/kernels/sgemm.cpp:23-27).
constexpr uint32_t kTcGemmAbi = 8;
constexpr int kMaxPeers = 7;  // one process per GPU, eight GPUs per node

enum TcKind : int { kKindF16 = 0, kKindI8 = 1, kKindF8 = 2 };
enum TcOut : int { kOutF32 = 0, kOutBF16 = 1, kOutF16 = 2, kOutS32 = 3 };

struct TcGemmParams {
  uint32_t abi_version;
  int m, n, k, batch;
  int a_mn_major, b_mn_major;      // smem layout of each operand
  int a_batch_step, b_batch_step;  // 1: batch coordinate walks the tensor map, 0: broadcast
  int m_tiles, n_tiles, k_blocks;
  int group_m;                     // rasterisation band height in m-tiles
  int tile_n;                      // single-CTA kernel: output columns per tile (32..256, see launch_tc_gemm)
  uint32_t idesc;                  // tcgen05 instruction descriptor
  float alpha, beta;
  int ialpha, ibeta;               // int32 epilogue (exact int8 path)
  int beta_nonzero;
  void* c;
  long long ldc, stride_c;
  const void* bias;
  int bias_bf16;
  int bias_rows;                   // 1: bias indexed by row i, 0: by column j
  int act;                         // grxblasActivation_t
  long long stride_bias;
  int scale_mode;                  // 0 none, 1 per-tensor, 2 per-row/per-column
  const float* scale_a;
  const float* scale_b;
  long long stride_sa, stride_sb;
  int* err_word;
  unsigned long long timeout_ns;
  // Tail split-K schedule. Tiles [0, sk_dp_tiles) run whole; each of the
  // next sk_tiles tiles is cut into sk_splits equal k-ranges, run as separate
  // units. Per epilogue warp (32 rows x 128 columns), the last unit of a cut
  // tile to arrive on sk_count[(tile - sk_dp_tiles) * 8 + warp] sums the
  // fp32/int32 partials of all splits (sk_part, one 128 x 256 slot per unit)
  // in split order, then runs the epilogue. sk_tiles == 0: whole tiles only.
  int sk_dp_tiles;
  int sk_tiles;
  int sk_splits;
  uint32_t* sk_part;
  int* sk_count;
  // Implicit-GEMM conv2d (conv != 0): op(A) is the K x (R S C) filter matrix,
  // op(B) the im2col of an NHWC input read by 4-D TMA loads, and tile column j
  // of n-tile nt is output pixel (img, p0 + j / cv_tw, q0 + j % cv_tw) of a
  // cv_th x cv_tw block (cv_th * cv_tw <= kTileN; later columns unused); C is
  // NHWC (ldc = K).
  int conv;
  int cv_p, cv_q, cv_th, cv_tw, cv_tiles_p, cv_tiles_q;
  int cv_sh, cv_sw, cv_ph, cv_pw, cv_dh, cv_dw, cv_s, cv_cb;
  uint32_t cv_b_bytes;  // bytes one pixel-block box delivers (th * tw * 128)
  // Replicated output: every element stored to c is also stored at the same
  // offset in peers[0 .. n_peers) (other GPUs' buffers opened in this process).
  int n_peers;
  void* peers[kMaxPeers];
  // Cycle probe (grxblasSetCycleProbe): when set, thread 0 of CTA b writes
  // probe[b] (clock64 at entry and exit, %smid, b). The host checks that
  // probe_capacity covers the grid before launching.
  grxCycleSlot* probe;
  int probe_capacity;
};

struct TcGemmLaunch {
  int kind;       // TcKind
  int out;        // TcOut
  int a_fmt;      // tcgen05 operand format code (f16 kind: 0 fp16, 1 bf16; i8: 1 signed; f8: 0 e4m3)
  // Operand storage: element (r, kk) of op(X) at base + b*stride + (mn_major ? r + kk*ld : kk + r*ld)
  const void* a; long long lda, stride_a; int a_mn_major;
  const void* b; long long ldb, stride_b; int b_mn_major;
  TcGemmParams p;
  // Device scratch for a split-K tail (tc_gemm_splitk_bytes); null or too
  // small: the launch keeps the whole-tile schedule.
  void* sk_ws;
  size_t sk_ws_bytes;
};

// Tile geometry shared by host and device.
constexpr int kTileM = 128;
constexpr int kTileN = 256;
constexpr int kStages = 4;
constexpr int kStageBytesA = kTileM * 128;   // 128 bytes of k per row
constexpr int kStageBytesB = kTileN * 128;
constexpr int kEpiWarps = 8;                      // two per TMEM lane quadrant, one per column half
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;  // warps: TMA, MMA, 8 x epilogue
constexpr int kGemmSmem = kStages * (kStageBytesA + kStageBytesB) + 1024 /*align*/ + 256 /*barriers*/;
// Most k-splits of one tile (bounds the planner).
constexpr int kSkMaxSeg = 8;

// CTA-pair (cta_group::2) variant: a cluster of 2 CTAs computes a 256 x 256
// tile; each CTA stages 128 rows of A and 128 columns of B per k-slab.
constexpr int kPairTileM = 256;
constexpr int kPairTileN = 256;
constexpr int kPairStages = 6;
constexpr int kPairStageBytes = 128 * 128;  // one operand half, 128 bytes of k per row
constexpr int kPairSmem = kPairStages * 2 * kPairStageBytes + 1024 + 256;

// Enqueues the kernel (builds the TMA tensor maps). Returns cudaErrorInvalidValue
// when an operand does not meet TMA alignment (the caller packs it first).
cudaError_t launch_tc_gemm(const TcGemmLaunch& L, int num_sms, cudaStream_t stream);

// Bytes of scratch the split-K tail of this problem wants (0: the problem
// runs as whole tiles). The decision matches launch_tc_gemm's.
size_t tc_gemm_splitk_bytes(int kind, int m, int n, int k, int batch, int num_sms);

// Implicit-GEMM conv2d on the tcgen05 kernel: x NHWC bf16 [n, h, w, c],
// filters KRSC bf16 [k, r, s, c], y NHWC [n, p, q, k] (bf16 or fp32 by out).
// Requires c % 64 == 0 and 16-byte aligned x / w. Epilogue: alpha, beta * y,
// bias over output channels (p.bias, bias_rows = 1) and p.act.
struct TcConvLaunch {
  int out;  // TcOut: kOutBF16 or kOutF32
  const void* x;
  const void* w;
  int n, h, wd, c, k, r, s, p, q;
  int pad_h, pad_w, stride_h, stride_w, dil_h, dil_w;
  TcGemmParams p_epi;  // alpha, beta, c, ldc, bias, act, err_word, timeout_ns
};
cudaError_t launch_tc_conv(const TcConvLaunch& L, int num_sms, cudaStream_t stream);

// True when an operand can be fed to TMA as stored.
bool tma_operand_ok(const void* base, long long ld, long long stride, int elem_bytes, int batch);

}  // namespace grx
