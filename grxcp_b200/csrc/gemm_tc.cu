// Tensor-core GEMM for sm_100a: tcgen05.mma with TMEM accumulators, fed by TMA
// through a multi-stage shared-memory ring, warp-specialised, persistent.
//
// Replaces the reference's hgemm_tcu / igemm_tcu kernels
// (src/libs/grxblas/kernels/hgemm_tcu.cpp:215-382), which walk 8x4x8 WMMA
// tiles from a single CTA. Semantics kept from there: column-major operands
// with all four transposes, C = alpha*acc + beta*C with beta == 0 never reading
// C (:354-357), the int8 epilogue in exact int32 arithmetic (:352-357), and
// masked edge tiles that never touch ld padding (:339-361).
//
// CTA organisation (320 threads, one CTA per SM, grid = min(tiles, SMs)):
//   warp 0      TMA producer: one thread streams A and B k-blocks into a
//               kStages-deep ring of 128-byte-swizzled smem stages.
//   warp 1      MMA issuer: one thread issues 4 tcgen05.mma per stage into a
//               128 x 256 fp32/int32 accumulator in TMEM and commits the stage
//               back to the producer; two accumulators (512 TMEM columns) let
//               the epilogue of tile i overlap the main loop of tile i+1.
//   warps 2..9  epilogue, two warps per TMEM lane quadrant (warp w reads lanes
//               32*(w%4).., columns of half (w-2)/4): tcgen05.ld 32 columns at
//               a time (thread = output row, so a warp's stores down a column
//               of C are contiguous), apply alpha / scales / beta*C / bias /
//               activation, convert, store. With one warp per SM
//               sub-partition the epilogue was latency-bound (about 9 cycles
//               per instruction, 16-20 us per tile); two per sub-partition
//               plus the pipelined TMEM reads cut that several-fold.
// Every mbarrier wait is bounded (ptx.cuh); a timeout aborts the CTA cleanly.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <stdlib.h>

#include <mutex>

#include "activation.cuh"
#include "gemm_tc.cuh"
#include "ptx.cuh"
#include "profile.h"

namespace grx {

__device__ __forceinline__ void decode_tile(const TcGemmParams& p, int t, int& bt, int& mt, int& nt) {
  const int tpb = p.m_tiles * p.n_tiles;
  bt = t / tpb;
  const int r = t - bt * tpb;
  const int group = p.group_m * p.n_tiles;
  const int g = r / group;
  const int first = g * p.group_m;
  const int gm = min(p.m_tiles - first, p.group_m);
  const int w = r - g * group;
  mt = first + w % gm;
  nt = w / gm;
}

// The work units of one CTA, in the order its producer, MMA issuer and
// epilogue all walk them (units blockIdx.x, blockIdx.x + gridDim.x, ...).
// Units [0, sk_dp_tiles) are whole tiles; unit sk_dp_tiles + v is k-range
// v / sk_tiles (of sk_splits equal ranges) of tile sk_dp_tiles + v % sk_tiles.
// Split-major order keeps the CTAs of one wave on the same k-range, so the A
// and B slabs they share are read from L2 together, as in the whole-tile
// schedule (a stream-K order, with each CTA on its own contiguous range of
// k-iterations, put concurrent CTAs at unrelated k offsets and re-read A from
// DRAM: 8192 x 1024 x 8192 went from 130 to 196 us). A unit is (tile,
// k-blocks [kb0, kb1), split; split -1 = whole tile).
struct WorkIter {
  int u, step;
  __device__ __forceinline__ WorkIter() : u(blockIdx.x), step(gridDim.x) {}
  // CTA-pair kernel: both CTAs of pair `first` walk the same units.
  __device__ __forceinline__ WorkIter(int first, int stride) : u(first), step(stride) {}
  __device__ __forceinline__ bool next(const TcGemmParams& p, int& tile, int& kb0, int& kb1, int& split) {
    const int units = p.sk_dp_tiles + p.sk_tiles * p.sk_splits;
    if (u >= units) return false;
    if (u < p.sk_dp_tiles) {
      tile = u;
      kb0 = 0;
      kb1 = p.k_blocks;
      split = -1;
    } else {
      const int v = u - p.sk_dp_tiles;
      split = v / p.sk_tiles;
      tile = p.sk_dp_tiles + (v - split * p.sk_tiles);
      kb0 = (int)((long long)split * p.k_blocks / p.sk_splits);
      kb1 = (int)((long long)(split + 1) * p.k_blocks / p.sk_splits);
    }
    u += step;
    return true;
  }
};

// Split-K partial slots. A slot holds one cut unit's 128 x 256 accumulator
// tile as 32-bit words ordered [column chunk c / 32][column group (c % 32) / 4]
// [row][c % 4]: a warp moves its 32 rows x 4 columns with one coalesced
// 512-byte access of 16 bytes per lane.
__device__ __forceinline__ size_t sk_slot_word(int chunk, int row) { return ((size_t)chunk * 8 * kTileM + row) * 4; }

// The partial accumulators of one cut tile as this epilogue thread sees them:
// split s left its tile in the slot at base + s * stride (words); split
// `self` is this unit's own, still in TMEM.
struct SkMerge {
  int n, self, row;
  const uint32_t* base;
  size_t stride;
};

template <int KIND>
__device__ __forceinline__ void sk_load(const SkMerge& mg, int s, int chunk, const uint32_t (&own)[32],
                                        uint32_t (&dst)[32]) {
  if (s == mg.self) {
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) dst[jj] = own[jj];
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(mg.base + s * mg.stride + sk_slot_word(chunk, mg.row));
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const uint4 w = __ldcg(src + g * kTileM);
    dst[4 * g] = w.x;
    dst[4 * g + 1] = w.y;
    dst[4 * g + 2] = w.z;
    dst[4 * g + 3] = w.w;
  }
}

// Replaces the 32 accumulators of chunk c0 by the sum over all splits, taken
// in split order whichever CTA reduces (so the result does not depend on
// arrival order): fp32 adds for the float kinds, int32 adds for i8.
template <int KIND>
__device__ __forceinline__ void sk_merge(const SkMerge& mg, int c0, uint32_t (&r)[32]) {
  const int chunk = c0 >> 5;
  uint32_t acc[32], v[32];
  sk_load<KIND>(mg, 0, chunk, r, acc);
#pragma unroll 1
  for (int s = 1; s < mg.n; ++s) {
    sk_load<KIND>(mg, s, chunk, r, v);
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      if (KIND == kKindI8) acc[jj] = (uint32_t)((int)acc[jj] + (int)v[jj]);
      else acc[jj] = __float_as_uint(__fadd_rn(__uint_as_float(acc[jj]), __uint_as_float(v[jj])));
    }
  }
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) r[jj] = acc[jj];
}

// The reducing warp's columns [cb, ce) of a cut tile: each 32-column chunk
// of its own accumulator is read from TMEM, replaced by the sum over all
// splits, and written back, so the ordinary epilogue then runs on the total.
template <int KIND>
__device__ __noinline__ void sk_reduce_into_tmem(const TcGemmParams& p, uint32_t t_row, const SkMerge& mg, int col0,
                                                    int cb, int ce) {
  for (int c0 = cb; c0 < ce; c0 += 32) {
    if (col0 + c0 >= p.n) break;  // warp-uniform
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c0, r);
    tmem_ld_wait_regs(r);
    sk_merge<KIND>(mg, c0, r);
    tmem_st_32x32b_x32(t_row + c0, r);
  }
  tmem_st_wait();
}

// This thread's row of a cut tile's accumulator, columns [cb, ce) of the tile,
// TMEM -> its partial slot.
__device__ __noinline__ void sk_store_partial(const TcGemmParams& p, uint32_t t_row, uint32_t* slot, int row,
                                                 int col0, int cb, int ce) {
  for (int c0 = cb; c0 < ce; c0 += 32) {
    if (col0 + c0 >= p.n) break;  // warp-uniform
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c0, r);
    tmem_ld_wait_regs(r);
    uint4* d = reinterpret_cast<uint4*>(slot + sk_slot_word(c0 >> 5, row));
#pragma unroll
    for (int g = 0; g < 8; ++g) __stcg(d + g * kTileM, make_uint4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]));
  }
}

// Output-pixel block of conv n-tile nt: image, first row, first column.
__device__ __forceinline__ void conv_tile(const TcGemmParams& p, int nt, int& img, int& p0, int& q0) {
  const int per_img = p.cv_tiles_p * p.cv_tiles_q;
  img = nt / per_img;
  const int rem = nt - img * per_img;
  const int tp = rem / p.cv_tiles_q;
  p0 = tp * p.cv_th;
  q0 = (rem - tp * p.cv_tiles_q) * p.cv_tw;
}

// Waits without honouring the abort flag: used only to let in-flight copies
// and MMAs land before the CTA releases its shared memory and TMEM.
static __device__ __noinline__ void wait_drain(uint64_t* bar, uint32_t parity, uint64_t timeout_ns, int* err) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      if (err) atomicCAS(err, 0, kErrTimeoutDrain);
      return;
    }
  }
}

template <int OUT>
__device__ __forceinline__ float load_c(const void* c, long long idx) {
  if constexpr (OUT == kOutF32) return static_cast<const float*>(c)[idx];
  else if constexpr (OUT == kOutBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(c)[idx]);
  else return __half2float(static_cast<const __half*>(c)[idx]);
}

template <int OUT>
__device__ __forceinline__ void store_c(void* c, long long idx, float v) {
  if constexpr (OUT == kOutF32) static_cast<float*>(c)[idx] = v;
  else if constexpr (OUT == kOutBF16) static_cast<__nv_bfloat16*>(c)[idx] = __float2bfloat16_rn(v);
  else static_cast<__half*>(c)[idx] = __float2half_rn(v);
}

// Epilogue of one output tile for the calling warp: 32 rows (thread = row i)
// x the 128 columns [cb, cb + 128) of the tile starting at column col0, read
// from TMEM at t_row 32 columns at a time. The next chunk's tcgen05.ld is in
// flight while the current chunk is converted and stored, and the per-column
// scale and bias of every chunk are loaded once up front.
//
// Fast path (a full 32 x 32 chunk, beta == 0, C and ldc allow 2-element
// stores): lanes 2r and 2r+1 swap one value with shfl.xor 1, so each lane
// holds two consecutive ROWS of one column -- adjacent in column-major C --
// and writes them with one 4-byte (16-bit C) or 8-byte (32-bit C) store; the
// scale / bias / activation choices are made once per chunk, not per
// element. Everything else (ragged edges, beta != 0) takes the element-wise
// path, which also defines the arithmetic both paths share.
// alpha * s(i,j) * acc, then (caller) + beta * C, then + bias[j].
template <int KIND>
__device__ __forceinline__ float epi_scaled(const TcGemmParams& p, uint32_t raw, float rowmul, const float* sb, int j) {
  const float acc = (KIND == kKindI8) ? (float)(int)raw : __uint_as_float(raw);
  float v = __fmul_rn(rowmul, acc);
  if (p.scale_mode == 2) v = __fmul_rn(v, sb[j]);
  return v;
}
// + bias (over columns j, or the row's value bias_row), then the activation.
__device__ __forceinline__ float epi_bias(const TcGemmParams& p, float v, const float* bias_f,
                                          const __nv_bfloat16* bias_h, int j, float bias_row) {
  if (p.bias) v = __fadd_rn(v, p.bias_rows ? bias_row : (p.bias_bf16 ? __bfloat162float(bias_h[j]) : bias_f[j]));
  return apply_act(v, p.act);
}

template <int ACT>
__device__ __forceinline__ void act_chunk(float (&v)[32]) {
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) v[jj] = apply_act(v[jj], ACT);
}

// Row-invariant state of one thread's row of the tile.
struct EpiRow {
  long long cbase;   // element index of (row i, column 0) of this batch member's C
  float rowmul;      // alpha times the row's scale
  float bias_row;
  bool row_ok, pair_ok;
};

// ncol: how many of the chunk's 32 columns exist (the rest are not stored).
// MASKED: the pair-store path takes partial chunks too (conv); otherwise it
// takes full chunks only and partial ones go element by element (GEMM).
// PEER: every value stored to C is stored at the same offset in each of the
// p.n_peers peer buffers too (plain stores over NVLink into other GPUs' C).
template <int KIND, int OUT, bool MASKED = false, bool PEER = false>
__device__ __forceinline__ void epi_chunk(const TcGemmParams& p, const EpiRow& er, uint32_t (&r)[32], int jbase,
                                          int ncol, float sb_l, float bias_l, const float* sb, const float* bias_f,
                                          const __nv_bfloat16* bias_h) {
  const int lane = threadIdx.x & 31;
  if (er.pair_ok && (MASKED || ncol == 32)) {
    const bool odd = lane & 1;
    // even lane: rows (i, i+1) of columns jbase+jj; odd lane: rows (i-1, i) of jbase+jj+1
    const long long base = er.cbase - (odd ? 1 : 0) + (long long)(jbase + (odd ? 1 : 0)) * p.ldc;
    const long long step = 2 * p.ldc;
    if constexpr (OUT == kOutS32) {
      int* cp = static_cast<int*>(p.c) + base;
#pragma unroll
      for (int jj = 0; jj < 32; jj += 2) {
        const int a = p.ialpha * (int)r[jj], b = p.ialpha * (int)r[jj + 1];
        const int other = __shfl_xor_sync(0xffffffffu, odd ? a : b, 1);
        if (!MASKED || jj + (odd ? 1 : 0) < ncol)
          *reinterpret_cast<int2*>(cp) = odd ? make_int2(other, b) : make_int2(a, other);
        cp += step;
      }
    } else {
      float v[32];
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        v[jj] = __fmul_rn(er.rowmul, (KIND == kKindI8) ? (float)(int)r[jj] : __uint_as_float(r[jj]));
      if (p.scale_mode == 2) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) v[jj] = __fmul_rn(v[jj], __shfl_sync(0xffffffffu, sb_l, jj));
      }
      if (p.bias) {
        if (p.bias_rows) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) v[jj] = __fadd_rn(v[jj], er.bias_row);
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) v[jj] = __fadd_rn(v[jj], __shfl_sync(0xffffffffu, bias_l, jj));
        }
      }
      switch (p.act) {
        case kActRelu: act_chunk<kActRelu>(v); break;
        case kActGeluTanh: act_chunk<kActGeluTanh>(v); break;
        case kActGeluErf: act_chunk<kActGeluErf>(v); break;
        default: break;
      }
#pragma unroll
      for (int jj = 0; jj < 32; jj += 2) {
        const float a = v[jj], b = v[jj + 1];
        const float other = __shfl_xor_sync(0xffffffffu, odd ? a : b, 1);
        const float lo = odd ? other : a, hi = odd ? b : other;  // lower row first
        const long long off = base + (long long)(jj / 2) * step;
        if (MASKED && jj + (odd ? 1 : 0) >= ncol) continue;
        if constexpr (OUT == kOutF32) {
          const float2 w = make_float2(lo, hi);
          *reinterpret_cast<float2*>(static_cast<float*>(p.c) + off) = w;
          if constexpr (PEER)
            for (int pr = 0; pr < p.n_peers; ++pr) *reinterpret_cast<float2*>(static_cast<float*>(p.peers[pr]) + off) = w;
        } else if constexpr (OUT == kOutBF16) {
          const __nv_bfloat162 w = __floats2bfloat162_rn(lo, hi);
          *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(p.c) + off) = w;
          if constexpr (PEER)
            for (int pr = 0; pr < p.n_peers; ++pr)
              *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(p.peers[pr]) + off) = w;
        } else {
          const __half2 w = __floats2half2_rn(lo, hi);
          *reinterpret_cast<__half2*>(static_cast<__half*>(p.c) + off) = w;
          if constexpr (PEER)
            for (int pr = 0; pr < p.n_peers; ++pr) *reinterpret_cast<__half2*>(static_cast<__half*>(p.peers[pr]) + off) = w;
        }
      }
    }
    return;
  }
  if (!er.row_ok) return;
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) {
    const int j = jbase + jj;
    if (jj < ncol) {
      const long long idx = er.cbase + (long long)j * p.ldc;
      if constexpr (OUT == kOutS32) {
        int v = p.ialpha * (int)r[jj];
        if (p.beta_nonzero) v += p.ibeta * static_cast<const int*>(p.c)[idx];
        static_cast<int*>(p.c)[idx] = v;
      } else {
        float v = epi_scaled<KIND>(p, r[jj], er.rowmul, sb, j);
        if (p.beta_nonzero) v = __fadd_rn(v, __fmul_rn(p.beta, load_c<OUT>(p.c, idx)));
        v = epi_bias(p, v, bias_f, bias_h, j, er.bias_row);
        store_c<OUT>(p.c, idx, v);
        if constexpr (PEER)
          for (int pr = 0; pr < p.n_peers; ++pr) store_c<OUT>(p.peers[pr], idx, v);
      }
    }
  }
}

constexpr int kEpiChunks = kTileN / 2 / 32;  // chunks of one epilogue warp's column half

template <int KIND, int OUT, bool PEER = false>
__device__ __forceinline__ void epilogue_tile(const TcGemmParams& p, uint32_t t_row, int bt, int i, int col0, int cb,
                                              int width = kTileN) {
  constexpr int kOutBytes = (OUT == kOutBF16 || OUT == kOutF16) ? 2 : 4;
  const int lane = threadIdx.x & 31;
  int cols = min(p.n - col0, width) - cb;
  if (cols > kEpiChunks * 32) cols = kEpiChunks * 32;
  const int nch = (cols + 31) / 32;
  if (nch <= 0) return;  // warp-uniform
  EpiRow er;
  er.row_ok = i < p.m;
  er.cbase = (long long)bt * p.stride_c + i;
  er.rowmul = p.alpha;
  if (p.scale_mode == 1) er.rowmul *= p.scale_a[bt * p.stride_sa] * p.scale_b[bt * p.stride_sb];
  if (p.scale_mode == 2 && er.row_ok) er.rowmul *= p.scale_a[bt * p.stride_sa + i];
  const float* sb = p.scale_b + bt * p.stride_sb;
  const float* bias_f = static_cast<const float*>(p.bias) + bt * p.stride_bias;
  const __nv_bfloat16* bias_h = static_cast<const __nv_bfloat16*>(p.bias) + bt * p.stride_bias;
  er.bias_row = (p.bias && p.bias_rows && er.row_ok) ? (p.bias_bf16 ? __bfloat162float(bias_h[i]) : bias_f[i]) : 0.f;
  // Pair stores need an even row index for the even lane, an even ldc / batch
  // stride and a C base aligned to two elements.
  const int i_warp0 = __shfl_sync(0xffffffffu, i, 0);
  er.pair_ok = !p.beta_nonzero && (p.ldc % 2 == 0) && (p.stride_c % 2 == 0) && (i_warp0 % 2 == 0) &&
               ((reinterpret_cast<uintptr_t>(p.c) % (2 * kOutBytes)) == 0) && i_warp0 + 31 < p.m;
  // This warp's column scales and biases: one value per lane per chunk,
  // broadcast by shuffle in the fast path.
  float sb_pre[kEpiChunks], bias_pre[kEpiChunks];
#pragma unroll
  for (int ci = 0; ci < kEpiChunks; ++ci) {
    const int j = col0 + cb + ci * 32 + lane;
    const bool ok = ci < nch && j < p.n;
    sb_pre[ci] = (p.scale_mode == 2 && ok) ? sb[j] : 1.f;
    bias_pre[ci] = (p.bias && !p.bias_rows && ok) ? (p.bias_bf16 ? __bfloat162float(bias_h[j]) : bias_f[j]) : 0.f;
  }
  uint32_t ra[32], rb[32];
  tmem_ld_32x32b_x32(t_row + cb, ra);
#pragma unroll
  for (int ci = 0; ci < kEpiChunks; ci += 2) {
    if (ci >= nch) break;
    tmem_ld_wait_regs(ra);
    if (ci + 1 < nch) tmem_ld_32x32b_x32(t_row + cb + (ci + 1) * 32, rb);
    epi_chunk<KIND, OUT, false, PEER>(p, er, ra, col0 + cb + ci * 32, min(32, p.n - (col0 + cb + ci * 32)), sb_pre[ci],
                         bias_pre[ci], sb, bias_f, bias_h);
    if (ci + 1 < nch) {
      tmem_ld_wait_regs(rb);
      if (ci + 2 < nch) tmem_ld_32x32b_x32(t_row + cb + (ci + 2) * 32, ra);
      epi_chunk<KIND, OUT, false, PEER>(p, er, rb, col0 + cb + (ci + 1) * 32, min(32, p.n - (col0 + cb + (ci + 1) * 32)),
                           sb_pre[ci + 1], bias_pre[ci + 1], sb, bias_f, bias_h);
    }
  }
}

// Conv epilogue: thread = output channel i, tile column j = output pixel.
// Full-row blocks (cv_tw == output width): the tile is one contiguous run of
// output pixels. Wide rows (cv_tw a multiple of 32 below the output width):
// each 32-column chunk lies in one output row. Either way a chunk is up to 32
// consecutive NHWC pixels (stride ldc), stored through the GEMM chunk path
// with pair stores over adjacent channels.
template <int KIND, int OUT>
__device__ __forceinline__ void epilogue_conv(const TcGemmParams& p, uint32_t t_row, int i, int nt, int cb) {
  constexpr int kOutBytes = (OUT == kOutBF16 || OUT == kOutF16) ? 2 : 4;
  int img, p0, q0;
  conv_tile(p, nt, img, p0, q0);
  const float* bias_f = static_cast<const float*>(p.bias);
  EpiRow er;
  er.row_ok = i < p.m;
  er.rowmul = p.alpha;
  er.bias_row = (p.bias && er.row_ok) ? bias_f[i] : 0.f;
  const int i_warp0 = __shfl_sync(0xffffffffu, i, 0);
  er.pair_ok = !p.beta_nonzero && (p.ldc % 2 == 0) && (i_warp0 % 2 == 0) &&
               ((reinterpret_cast<uintptr_t>(p.c) % (2 * kOutBytes)) == 0) && i_warp0 + 31 < p.m;
  const int rows_here = min(p.cv_th, p.cv_p - p0);
  for (int c0 = cb; c0 < cb + kTileN / 2; c0 += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c0, r);
    tmem_ld_wait_regs(r);
    int ncol;
    long long pix;
    if (p.cv_tw == p.cv_q) {
      ncol = min(32, rows_here * p.cv_q - c0);
      pix = ((long long)img * p.cv_p + p0) * p.cv_q + c0;
    } else {
      const int dp = c0 / p.cv_tw;
      const int qq = q0 + (c0 - dp * p.cv_tw);
      ncol = dp < rows_here ? min(32, p.cv_q - qq) : 0;
      pix = ((long long)img * p.cv_p + p0 + dp) * p.cv_q + qq;
    }
    if (ncol <= 0) continue;  // warp-uniform
    er.cbase = pix * p.ldc + i;
    epi_chunk<KIND, OUT, true>(p, er, r, 0, ncol, 1.f, 0.f, nullptr, bias_f, nullptr);
  }
}

// Cycle-probe record of this CTA (grxblasSetCycleProbe); thread 0 only.
__device__ __forceinline__ void probe_write(const TcGemmParams& p, uint64_t t0) {
  if (p.probe == nullptr || threadIdx.x != 0 || (int)blockIdx.x >= p.probe_capacity) return;
  unsigned smid;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
  grxCycleSlot s;
  s.start = t0;
  s.end = (uint64_t)clock64();
  s.core = smid;
  s.warp = blockIdx.x;
  p.probe[blockIdx.x] = s;
}

template <int KIND, int OUT, bool CONV, bool PEER>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ TcGemmParams p) {
  constexpr int ES = (KIND == kKindF16) ? 2 : 1;  // element bytes
  constexpr int BK = 128 / ES;                    // k per stage (one 128-byte swizzle row)
  constexpr int UK = 32 / ES;                     // k per tcgen05.mma
  constexpr int KSUB = BK / UK;                   // MMAs per stage
  constexpr int ATOM = 128 / ES;                  // elements in one MN-major swizzle row
  // Output columns per tile: kTileN, or fewer for problems with fewer tiles
  // than SMs (launch_tc_gemm); the B box then holds TN rows (K-major) or
  // TN / ATOM atoms (MN-major) and the MMA runs with N = TN.
  const int TN = CONV ? kTileN : p.tile_n;

  if (p.abi_version != kTcGemmAbi) {
    if (threadIdx.x == 0 && p.err_word) atomicCAS(p.err_word, 0, kErrBadAbi);
    return;
  }
  const uint64_t probe_t0 = p.probe ? clock64() : 0ull;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kStageBytesA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * kStageBytesB);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kTileN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  WaitCtx wc{p.err_word, abort_flag, p.timeout_ns};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_par = 0;
      bool ok = true;
      WorkIter it;
      int t, kb0, kb1, split;
      while (ok && it.next(p, t, kb0, kb1, split)) {
        int bt, mt, nt;
        decode_tile(p, t, bt, mt, nt);
        const int ba = bt * p.a_batch_step, bb = bt * p.b_batch_step;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(&empty[stage], phase ^ 1u, wc, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint64_t* fb = &full[stage];
          mbar_arrive_expect_tx(fb, CONV ? (uint32_t)kStageBytesA + p.cv_b_bytes : (uint32_t)(kStageBytesA + TN * 128));
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          uint8_t* a_dst = sA + stage * kStageBytesA;
          uint8_t* b_dst = sB + stage * kStageBytesB;
          const int k0 = kb * BK;
          if (!p.a_mn_major) {
            tma_load_3d(a_dst, &tmA, fb, k0, mt * kTileM, ba);
          } else {
#pragma unroll
            for (int j = 0; j < kTileM / ATOM; ++j)
              tma_load_3d(a_dst + j * (BK * 128), &tmA, fb, mt * kTileM + j * ATOM, k0, ba);
          }
          if constexpr (CONV) {
            // k-block kb = (filter tap r s, 64-channel block); the box of
            // cv_th x cv_tw output pixels reads input rows/columns at the
            // conv strides, and out-of-range (padding) coordinates read 0.
            const int rs = kb / p.cv_cb;
            const int c0 = (kb - rs * p.cv_cb) * 64;
            const int fr = rs / p.cv_s, fs = rs - fr * p.cv_s;
            int img, p0, q0;
            conv_tile(p, nt, img, p0, q0);
            tma_load_4d(b_dst, &tmB, fb, c0, q0 * p.cv_sw - p.cv_pw + fs * p.cv_dw,
                        p0 * p.cv_sh - p.cv_ph + fr * p.cv_dh, img);
          } else if (!p.b_mn_major) {
            tma_load_3d(b_dst, &tmB, fb, k0, nt * TN, bb);
          } else {
            for (int j = 0; j < TN / ATOM; ++j)
              tma_load_3d(b_dst + j * (BK * 128), &tmB, fb, nt * TN + j * ATOM, k0, bb);
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Let every armed stage land before the CTA's shared memory goes away:
      // after an abort elsewhere in the CTA (the MMA issuer stops consuming)
      // the last loads may still be in flight even though this loop finished.
      // On a normal exit every stage's last phase has completed already.
      for (int s = 0; s < kStages; ++s)
        if (issued_mask & (1u << s)) wait_drain(&full[s], (issued_par >> s) & 1u, p.timeout_ns, p.err_word);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      WorkIter it;
      int t, kb0, kb1, split;
      for (; ok && it.next(p, t, kb0, kb1, split); ++local) {
        const int b = local & 1;
        if (!wait_bounded(&tempty[b], ((local >> 1) & 1) ^ 1u, wc, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * kTileN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(&full[stage], phase, wc, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * kStageBytesA);
          const uint32_t b_addr = smem_u32(sB + stage * kStageBytesB);
#pragma unroll
          for (int kk = 0; kk < KSUB; ++kk) {
            const uint64_t ad = p.a_mn_major ? sw128_desc(a_addr + kk * UK * 128, BK * 128, 1024)
                                             : sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = p.b_mn_major ? sw128_desc(b_addr + kk * UK * 128, BK * 128, 1024)
                                             : sw128_desc(b_addr + kk * 32, 16, 1024);
            mma_ss<KIND>(d_tmem, ad, bd, p.idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[b]);
      }
      // Every MMA this thread issued must complete before TMEM is released.
      mma_commit(drain);
      wait_drain(drain, 0, p.timeout_ns, p.err_word);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                           // TMEM lane quadrant this warp may access
    const int cb = ((warp - 2) >> 2) * (kTileN / 2);  // its column half
    const int row = q * 32 + lane;
    int local = 0;
    WorkIter it;
    int t, kb0, kb1, split;
    for (; it.next(p, t, kb0, kb1, split); ++local) {
      const int b = local & 1;
      if (!wait_bounded(&tfull[b], (local >> 1) & 1, wc, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      int bt, mt, nt;
      decode_tile(p, t, bt, mt, nt);
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + b * kTileN;
      if constexpr (CONV) {
        epilogue_conv<KIND, OUT>(p, t_row, mt * kTileM + row, nt, cb);
      } else if (split < 0) {
        epilogue_tile<KIND, OUT, PEER>(p, t_row, bt, mt * kTileM + row, nt * TN, cb, TN);
      } else {
        // A cut tile: publish this unit's partial, count it in, and let the
        // last split of the tile to arrive reduce and write C. Nobody waits on
        // another CTA, so the schedule needs no co-residency. Each warp owns
        // its 32 rows x 128 columns end to end, with one arrival counter per
        // (tile, epilogue warp): no barrier between warps.
        const int r = t - p.sk_dp_tiles;
        SkMerge mg;
        mg.n = p.sk_splits;
        mg.self = split;
        mg.row = row;
        mg.stride = (size_t)p.sk_tiles * (kTileN * kTileM);
        mg.base = p.sk_part + (size_t)r * (kTileN * kTileM);
        int* count = p.sk_count + (size_t)r * kEpiWarps + (warp - 2);
        // The last split normally runs after all the others have arrived
        // (units go split-major); it then reduces from its own TMEM without
        // publishing. Otherwise it publishes and counts in like the rest.
        int before = 0;
        if (split == mg.n - 1) {
          if (lane == 0) before = ld_acquire_gpu(count);
          before = __shfl_sync(0xffffffffu, before, 0);
        }
        if (before != mg.n - 1) {
          sk_store_partial(p, t_row, p.sk_part + (size_t)r * (kTileN * kTileM) + split * mg.stride, row,
                           nt * kTileN, cb, cb + kTileN / 2);
          __threadfence();
          __syncwarp();
          if (lane == 0) before = atomicAdd(count, 1);
          before = __shfl_sync(0xffffffffu, before, 0);
        }
        if (before == mg.n - 1) {
          __threadfence();
          sk_reduce_into_tmem<KIND>(p, t_row, mg, nt * kTileN, cb, cb + kTileN / 2);
          epilogue_tile<KIND, OUT, PEER>(p, t_row, bt, mt * kTileM + row, nt * kTileN, cb);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if constexpr (PEER) __threadfence_system();  // this thread's stores into peer GPUs' C are performed
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kTileN);
  }
  probe_write(p, probe_t0);
}

// CTA-pair kernel. Cluster of two CTAs (rank 0 = leader). Each CTA:
//   warp 0      streams its 128 rows of A and its 128 columns of B per k-slab
//               into its own kPairStages-deep ring; completion bytes of both
//               CTAs are counted on the leader's full barrier.
//   warp 1      leader only: one thread issues tcgen05.mma.cta_group::2
//               (M = 256 over both CTAs' rows, N = 256 over both CTAs' B
//               halves), and commits each stage / accumulator to the
//               barriers of both CTAs.
//   warps 2..9  epilogue of this CTA's 128 rows x 256 columns from its own
//               TMEM, then one arrival on the leader's accumulator-free barrier.
// Per SM this halves the B bytes per FLOP of the single-CTA kernel, so the
// same shared memory keeps the tensor pipe fed across longer L2 latency.
template <int KIND, int OUT, bool PEER>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ TcGemmParams p) {
  constexpr int ES = (KIND == kKindF16) ? 2 : 1;
  constexpr int BK = 128 / ES;
  constexpr int UK = 32 / ES;
  constexpr int KSUB = BK / UK;
  constexpr int ATOM = 128 / ES;
  constexpr uint32_t kStageTx = 2u * 2u * kPairStageBytes;  // A + B halves of both CTAs

  if (p.abi_version != kTcGemmAbi) {
    if (threadIdx.x == 0 && p.err_word) atomicCAS(p.err_word, 0, kErrBadAbi);
    return;  // both CTAs of every pair take this branch alike
  }
  const uint64_t probe_t0 = p.probe ? clock64() : 0ull;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kPairStages * kPairStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kPairStages * kPairStageBytes);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);  // epilogue warps of both CTAs (used on the leader)
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * kPairTileN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  WaitCtx wc{p.err_word, abort_flag, p.timeout_ns};
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      WorkIter it(pair, npairs);
      int t, kb0, kb1, split;
      while (ok && it.next(p, t, kb0, kb1, split)) {
        int bt, mt, nt;
        decode_tile(p, t, bt, mt, nt);
        const int ba = bt * p.a_batch_step, bb = bt * p.b_batch_step;
        const int row0 = mt * kPairTileM + (int)rank * 128;
        const int col0 = nt * kPairTileN + (int)rank * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(&empty[stage], phase ^ 1u, wc, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) {
            mbar_arrive_expect_tx(&full[stage], kStageTx);
            armed |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t fb = leader_addr(&full[stage]);
          uint8_t* a_dst = sA + stage * kPairStageBytes;
          uint8_t* b_dst = sB + stage * kPairStageBytes;
          const int k0 = kb * BK;
          if (!p.a_mn_major) {
            tma_load_3d_pair(a_dst, &tmA, fb, k0, row0, ba);
          } else {
#pragma unroll
            for (int j = 0; j < 128 / ATOM; ++j) tma_load_3d_pair(a_dst + j * (BK * 128), &tmA, fb, row0 + j * ATOM, k0, ba);
          }
          if (!p.b_mn_major) {
            tma_load_3d_pair(b_dst, &tmB, fb, k0, col0, bb);
          } else {
#pragma unroll
            for (int j = 0; j < 128 / ATOM; ++j) tma_load_3d_pair(b_dst + j * (BK * 128), &tmB, fb, col0 + j * ATOM, k0, bb);
          }
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Both CTAs' loads complete on the leader's full barriers: after an
      // abort the leader lets every armed stage land; the closing cluster
      // barrier holds the peer until then.
      if (leader) {
        for (int s = 0; s < kPairStages; ++s)
          if (armed & (1u << s)) wait_drain(&full[s], (armed_par >> s) & 1u, p.timeout_ns, p.err_word);
      }
      // After an abort the peer CTA may have issued loads (completing on the
      // leader's barriers) for stages the leader never armed; give copies in
      // flight time to land before either CTA's shared memory is released.
      if (*abort_flag) {
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 50000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      WorkIter it(pair, npairs);
      int t, kb0, kb1, split;
      for (; ok && it.next(p, t, kb0, kb1, split); ++local) {
        const int b = local & 1;
        if (!wait_bounded(&tempty[b], ((local >> 1) & 1) ^ 1u, wc, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * kPairTileN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(&full[stage], phase, wc, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * kPairStageBytes);
          const uint32_t b_addr = smem_u32(sB + stage * kPairStageBytes);
#pragma unroll
          for (int kk = 0; kk < KSUB; ++kk) {
            const uint64_t ad = p.a_mn_major ? sw128_desc(a_addr + kk * UK * 128, BK * 128, 1024)
                                             : sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = p.b_mn_major ? sw128_desc(b_addr + kk * UK * 128, BK * 128, 1024)
                                             : sw128_desc(b_addr + kk * 32, 16, 1024);
            mma_ss_pair<KIND>(d_tmem, ad, bd, p.idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(&tfull[b], 0x3);
      }
      mma_commit_pair(drain, 0x1);
      wait_drain(drain, 0, p.timeout_ns, p.err_word);
    }
  } else {
    const int q = warp & 3;
    const int cb = ((warp - 2) >> 2) * (kPairTileN / 2);
    const int row = q * 32 + lane;
    int local = 0;
    WorkIter it(pair, npairs);
    int t, kb0, kb1, split;
    for (; it.next(p, t, kb0, kb1, split); ++local) {
      const int b = local & 1;
      if (!wait_bounded(&tfull[b], (local >> 1) & 1, wc, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      int bt, mt, nt;
      decode_tile(p, t, bt, mt, nt);
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + b * kPairTileN;
      const int grow = mt * kPairTileM + (int)rank * 128 + row;
      bool write_c = true;
      if (split >= 0) {
        // A cut tile, as in the single-CTA kernel, per CTA half: each CTA of the
        // pair owns its own 128 x 256 partial slot (slot (tile - dp) * 2 + rank)
        // and arrival counter per epilogue warp; the last split to arrive sums
        // all splits in split order and writes C.
        const int r = (t - p.sk_dp_tiles) * 2 + (int)rank;
        SkMerge mg;
        mg.n = p.sk_splits;
        mg.self = split;
        mg.row = row;
        mg.stride = (size_t)p.sk_tiles * 2 * (kTileN * kTileM);
        mg.base = p.sk_part + (size_t)r * (kTileN * kTileM);
        int* count = p.sk_count + (size_t)r * kEpiWarps + (warp - 2);
        int before = 0;
        if (split == mg.n - 1) {
          if (lane == 0) before = ld_acquire_gpu(count);
          before = __shfl_sync(0xffffffffu, before, 0);
        }
        if (before != mg.n - 1) {
          sk_store_partial(p, t_row, p.sk_part + (size_t)r * (kTileN * kTileM) + split * mg.stride, row,
                           nt * kPairTileN, cb, cb + kPairTileN / 2);
          __threadfence();
          __syncwarp();
          if (lane == 0) before = atomicAdd(count, 1);
          before = __shfl_sync(0xffffffffu, before, 0);
        }
        write_c = before == mg.n - 1;
        if (write_c) {
          __threadfence();
          sk_reduce_into_tmem<KIND>(p, t_row, mg, nt * kPairTileN, cb, cb + kPairTileN / 2);
        }
      }
      if (write_c) epilogue_tile<KIND, OUT, PEER>(p, t_row, bt, grow, nt * kPairTileN, cb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&tempty[b]);
        else mbar_arrive_cluster(&tempty[b], 0);
      }
    }
    if constexpr (PEER) __threadfence_system();  // this thread's stores into peer GPUs' C are performed
  }

  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still touch its smem or TMEM
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * kPairTileN);
  }
  probe_write(p, probe_t0);
}

// ---------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

bool tma_operand_ok(const void* base, long long ld, long long stride, int elem_bytes, int batch) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if ((ld * elem_bytes) % 16 != 0) return false;
  if (batch > 1 && stride != 0) {
    if (stride < 0) return false;
    if ((stride * elem_bytes) % 16 != 0) return false;
  }
  return true;
}

// Operand tensor map: K-major -> dims {K, MN, batch}, box {BK, tile};
// MN-major -> dims {MN, K, batch}, box {128 bytes of MN, BK}. 128-byte swizzle.
static bool make_operand_map(CUtensorMap* map, const void* base, int es, int mn_major, long long mn_extent,
                             long long k_extent, long long ld, long long stride, int batch_dim, int tile_mn) {
  const int bk = 128 / es;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3], estr[3] = {1, 1, 1};
  if (!mn_major) {
    dims[0] = (cuuint64_t)k_extent;
    dims[1] = (cuuint64_t)mn_extent;
    box[0] = bk;
    box[1] = tile_mn;
  } else {
    dims[0] = (cuuint64_t)mn_extent;
    dims[1] = (cuuint64_t)k_extent;
    box[0] = 128 / es;
    box[1] = bk;
  }
  dims[2] = (cuuint64_t)batch_dim;
  box[2] = 1;
  strides[0] = (cuuint64_t)(ld * es);
  strides[1] = batch_dim > 1 ? (cuuint64_t)(stride * es) : (cuuint64_t)(ld * es) * dims[1];
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const CUtensorMapDataType dt = es == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int KIND, int OUT, bool CONV = false, bool PEER = false>
static cudaError_t launch_impl(const CUtensorMap& ma, const CUtensorMap& mb, const TcGemmParams& p, int grid,
                               cudaStream_t s) {
  auto kfn = tc_gemm_kernel<KIND, OUT, CONV, PEER>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  });
  if (attr_err != cudaSuccess) return attr_err;
  ProfLaunch prof("tc_gemm_kernel", dim3(grid), dim3(kGemmThreads), kGemmSmem, s);
  kfn<<<grid, kGemmThreads, kGemmSmem, s>>>(ma, mb, p);
  return cudaGetLastError();
}

template <int KIND, int OUT, bool PEER = false>
static cudaError_t launch_pair_impl(const CUtensorMap& ma, const CUtensorMap& mb, const TcGemmParams& p, int grid,
                                    cudaStream_t s) {
  auto kfn = tc_gemm_pair_kernel<KIND, OUT, PEER>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem);
  });
  if (attr_err != cudaSuccess) return attr_err;
  ProfLaunch prof("tc_gemm_pair_kernel", dim3(grid), dim3(kGemmThreads), kPairSmem, s);
  kfn<<<grid, kGemmThreads, kPairSmem, s>>>(ma, mb, p);
  return cudaGetLastError();
}

// Measured on B200 (8192^3): the pair kernel wins for 16-bit operands with an
// MN-major operand (NN +8 %, NT +14 %, TT +2 %) and ties on TN; it loses for
// 8-bit operands (the tensor pipe consumes k twice as fast there, so the
// extra cross-CTA hand-off shows). With bf16 data of the bench's scale it
// also wins on the column-parallel slices once there is at least one pair
// tile per SM pair: 8192 x 2048 x 8192 215 vs 222 us, 8192 x 1024 x 8192 109
// vs 114 us, 18944 x 256 x 8192 (one round) 66 vs 73 us.
// GRX_GEMM_NO_PAIR=1 forces the single-CTA kernel; GRX_GEMM_FORCE_PAIR=1
// takes the pair kernel for every type whenever m and n are at least 256 (the
// tests use it to cover that kernel at modest sizes).
static bool use_pair(int kind, const TcGemmParams& p, int num_sms) {
  if (getenv("GRX_GEMM_NO_PAIR")) return false;
  if (getenv("GRX_GEMM_FORCE_PAIR")) return p.m >= kPairTileM && p.n >= kPairTileN;
  if (kind != kKindF16) return false;
  const long long tiles = (long long)((p.m + kPairTileM - 1) / kPairTileM) * ((p.n + kPairTileN - 1) / kPairTileN) *
                          p.batch;
  return p.m >= kPairTileM && p.n >= kPairTileN && tiles >= (long long)(num_sms / 2);
}

// Split-K plan for the last, partial wave of the single-CTA kernel. A
// whole-tile schedule of T tiles on S SMs runs ceil(T / S) waves of K
// k-blocks, the last with only R = T % S busy CTAs; with few waves that tail
// is a large share of the time (an 8192 x 1024 x 8192 bf16 slice is 256 tiles
// = 1.73 waves on 148 SMs). The plan keeps the floor(T / S) full waves whole
// and cuts each of the R tail tiles into s k-ranges, choosing s in 2..8 to
// minimise ceil(R s / S) * (ceil(K / s) + kSkWaveCost), the tail's length in
// k-blocks with an allowance per wave of cut units for publishing and summing
// the partials (about 11 us measured on B200, 24 k-blocks of a 128 x 256 x 64
// bf16 step); each range keeps at least 4 k-blocks, the partials take at most
// 64 MiB, and a plan must shorten the tail by at least 20 %. Measured on
// B200 against whole tiles: 1024 x 1024 x 8192 1.44x, 512 x 1024 x 8192
// 1.41x, 8192 x 1280 x 8192 1.10x, 8192 x 2048 x 8192 1.02x; shapes the plan
// leaves whole (8192 x 1024 x 8192: cutting 108 tail tiles four ways saves
// 20 k-blocks but costs three waves of overhead) run as before. GRX_GEMM_SPLITK=0 turns it off; GRX_GEMM_FORCE_SK=s cuts every tile
// into min(s, 8, K) ranges (the tests use it at modest sizes).
constexpr int kSkWaveCost = 24;

struct SkPlan {
  long long dp_tiles = 0, sk_tiles = 0;
  int splits = 1;
};

static bool plan_splitk(long long tiles, int k_blocks, int num_sms, SkPlan& sp) {
  if (const char* e = getenv("GRX_GEMM_SPLITK"))
    if (e[0] == '0') return false;
  if (tiles < 1 || k_blocks < 2 || num_sms < 1) return false;
  constexpr long long kMaxUnits = (64ll << 20) / (kTileM * kTileN * 4);
  if (const char* f = getenv("GRX_GEMM_FORCE_SK")) {
    int sf = atoi(f);
    if (sf > kSkMaxSeg) sf = kSkMaxSeg;
    if (sf > k_blocks) sf = k_blocks;
    if (sf < 2 || tiles * sf > kMaxUnits) return false;
    sp.dp_tiles = 0;
    sp.sk_tiles = tiles;
    sp.splits = sf;
    return true;
  }
  const long long rem = tiles % num_sms;
  if (rem == 0) return false;
  long long best = k_blocks;  // the whole-tile tail: one wave of K
  int best_s = 1;
  for (int sv = 2; sv <= kSkMaxSeg; ++sv) {
    if (k_blocks / sv < 4 || rem * sv > kMaxUnits) break;
    const long long cost = (rem * sv + num_sms - 1) / num_sms * ((k_blocks + sv - 1) / sv + kSkWaveCost);
    if (cost < best) {
      best = cost;
      best_s = sv;
    }
  }
  if (best_s == 1 || best * 10 > k_blocks * 8) return false;  // keep only plans that shorten the tail by >= 20 %
  sp.dp_tiles = tiles - rem;
  sp.sk_tiles = rem;
  sp.splits = best_s;
  return true;
}

// ctas = CTAs per tile (1, or 2 for the pair kernel: one partial slot and one
// set of counters per CTA).
static size_t splitk_bytes(const SkPlan& sp, int ctas = 1) {
  const size_t parts = (size_t)sp.sk_tiles * sp.splits * ctas * kTileM * kTileN * sizeof(uint32_t);
  const size_t counts = ((size_t)sp.sk_tiles * ctas * kEpiWarps * sizeof(int) + 255) & ~(size_t)255;
  return parts + counts;
}

size_t tc_gemm_splitk_bytes(int kind, int m, int n, int k, int batch, int num_sms) {
  if (m <= 0 || n <= 0 || k <= 0 || batch <= 0) return 0;
  TcGemmParams p{};
  p.m = m;
  p.n = n;
  p.batch = batch;
  const int bk = 128 / (kind == kKindF16 ? 2 : 1);
  SkPlan sp;
  if (use_pair(kind, p, num_sms)) {
    const long long pt = (long long)((m + kPairTileM - 1) / kPairTileM) * ((n + kPairTileN - 1) / kPairTileN) * batch;
    return plan_splitk(pt, (k + bk - 1) / bk, num_sms / 2, sp) ? splitk_bytes(sp, 2) : 0;
  }
  const long long tiles = (long long)((m + kTileM - 1) / kTileM) * ((n + kTileN - 1) / kTileN) * batch;
  return plan_splitk(tiles, (k + bk - 1) / bk, num_sms, sp) ? splitk_bytes(sp) : 0;
}

// NHWC bf16 input as a 4-D map {c, w, h, n}: box {64 channels, tw * sw
// columns, th * sh rows, 1 image} with traversal strides {1, sw, sh, 1}, so a
// load returns th x tw pixels x 64 channels, 128 bytes per pixel row of the
// 128-byte swizzle.
static bool make_conv_map(CUtensorMap* map, const void* x, int n, int h, int w, int c, int th, int tw, int sh,
                          int sw) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)c * 2, (cuuint64_t)w * c * 2, (cuuint64_t)h * w * c * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)(tw * sw), (cuuint32_t)(th * sh), 1};
  cuuint32_t estr[4] = {1, (cuuint32_t)sw, (cuuint32_t)sh, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_tc_conv(const TcConvLaunch& L, int num_sms, cudaStream_t stream) {
  if (L.c % 64 || (reinterpret_cast<uintptr_t>(L.x) & 15u) || (reinterpret_cast<uintptr_t>(L.w) & 15u))
    return cudaErrorNotSupported;
  if (L.stride_h < 1 || L.stride_w < 1 || L.stride_h > 8 || L.stride_w > 8) return cudaErrorNotSupported;
  // Pixel block of th x tw output pixels (th * tw <= kTileN columns). Whole
  // output rows when they fit the box (tw = q, th = 256 / q): the tile is
  // then one contiguous run of output pixels. Otherwise wide rows cut into
  // multiples of 32 columns. Each box dimension spans at most 256 input
  // elements (tw * stride_w, th * stride_h).
  int tw, th;
  if ((long long)L.q * L.stride_w <= 256) {
    tw = L.q;
    th = kTileN / tw;
  } else {
    tw = (256 / L.stride_w) & ~31;
    th = kTileN / tw;
  }
  if (th * L.stride_h > 256) th = 256 / L.stride_h;
  if (tw < 1 || th < 1) return cudaErrorNotSupported;
  TcGemmParams p = L.p_epi;
  p.abi_version = kTcGemmAbi;
  p.conv = 1;
  p.m = L.k;
  p.k = L.r * L.s * L.c;
  p.batch = 1;
  p.cv_p = L.p;
  p.cv_q = L.q;
  p.cv_th = th;
  p.cv_tw = tw;
  p.cv_tiles_p = (L.p + th - 1) / th;
  p.cv_tiles_q = (L.q + tw - 1) / tw;
  p.cv_sh = L.stride_h;
  p.cv_sw = L.stride_w;
  p.cv_ph = L.pad_h;
  p.cv_pw = L.pad_w;
  p.cv_dh = L.dil_h;
  p.cv_dw = L.dil_w;
  p.cv_s = L.s;
  p.cv_cb = L.c / 64;
  p.cv_b_bytes = (uint32_t)(128 * tw * th);
  p.n = L.n * L.p * L.q;
  p.m_tiles = (L.k + kTileM - 1) / kTileM;
  const long long n_tiles = (long long)L.n * p.cv_tiles_p * p.cv_tiles_q;
  const long long tiles = n_tiles * p.m_tiles;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  p.n_tiles = (int)n_tiles;
  p.k_blocks = p.k / 64;
  if (p.group_m <= 0) p.group_m = 16;
  p.a_mn_major = 0;
  p.b_mn_major = 0;
  p.a_batch_step = p.b_batch_step = 0;
  p.idesc = make_idesc(1u, 1u, 1u, 0u, 0u, kTileM, kTileN);
  p.tile_n = kTileN;
  p.sk_dp_tiles = (int)tiles;
  p.sk_tiles = 0;
  p.sk_splits = 1;
  CUtensorMap ma, mb;
  if (!make_operand_map(&ma, L.w, 2, 0, L.k, p.k, p.k, 0, 1, 128)) return cudaErrorNotSupported;
  if (!make_conv_map(&mb, L.x, L.n, L.h, L.wd, L.c, th, tw, L.stride_h, L.stride_w)) return cudaErrorNotSupported;
  const int grid = (int)(tiles < num_sms ? tiles : num_sms);
  if (L.out == kOutBF16) return launch_impl<kKindF16, kOutBF16, true>(ma, mb, p, grid, stream);
  if (L.out == kOutF32) return launch_impl<kKindF16, kOutF32, true>(ma, mb, p, grid, stream);
  return cudaErrorNotSupported;
}

cudaError_t launch_tc_gemm(const TcGemmLaunch& L, int num_sms, cudaStream_t stream) {
  const int es = L.kind == kKindF16 ? 2 : 1;
  TcGemmParams p = L.p;
  p.abi_version = kTcGemmAbi;
  const int bk = 128 / es;
  const bool pair = use_pair(L.kind, p, num_sms);
  const int tile_m = pair ? kPairTileM : kTileM;
  int tile_n = pair ? kPairTileN : kTileN;
  p.m_tiles = (p.m + tile_m - 1) / tile_m;
  p.n_tiles = (p.n + tile_n - 1) / tile_n;
  p.k_blocks = (p.k + bk - 1) / bk;
  // Single-CTA kernel: a split-K tail for few tiles with long K; otherwise,
  // while the tiles fill at most half the SMs, halve the tile's columns (down
  // to 32; an MN-major B keeps whole 128-byte atoms) so more SMs share the
  // MMAs and, above all, the epilogue's stores (int8 512^3:
  // 8 CTAs of 128 x 256 become 64 of 128 x 32).
  SkPlan sp;
  bool splitk = false;
  if (!pair) {
    const long long tiles256 = (long long)p.m_tiles * p.n_tiles * p.batch;
    splitk = L.sk_ws && plan_splitk(tiles256, p.k_blocks, num_sms, sp) && L.sk_ws_bytes >= splitk_bytes(sp);
    const int min_tn = L.b_mn_major ? 128 / es : 32;
    if (!splitk && !getenv("GRX_GEMM_WIDE_TILES")) {
      while (tile_n / 2 >= min_tn) {
        const long long t2 = (long long)p.m_tiles * ((p.n + tile_n / 2 - 1) / (tile_n / 2)) * p.batch;
        if (t2 > num_sms) break;
        tile_n /= 2;
      }
      p.n_tiles = (p.n + tile_n - 1) / tile_n;
    }
  }
  p.tile_n = tile_n;
  if (p.group_m <= 0) p.group_m = 16;
  p.a_mn_major = L.a_mn_major;
  p.b_mn_major = L.b_mn_major;
  // kind::i8 accumulates in s32 only (f32 is an illegal instruction there); the
  // epilogue converts to the requested output type.
  const uint32_t cfmt = (L.kind == kKindI8) ? 2u : 1u;
  p.idesc = make_idesc(cfmt, (uint32_t)L.a_fmt, (uint32_t)L.a_fmt, (uint32_t)L.a_mn_major, (uint32_t)L.b_mn_major,
                       pair ? kPairTileM : kTileM, pair ? kPairTileN : tile_n);
  const int a_bdim = (p.batch > 1 && L.stride_a != 0) ? p.batch : 1;
  const int b_bdim = (p.batch > 1 && L.stride_b != 0) ? p.batch : 1;
  p.a_batch_step = a_bdim > 1 ? 1 : 0;
  p.b_batch_step = b_bdim > 1 ? 1 : 0;
  CUtensorMap ma, mb;
  // Box rows: 128 of A per CTA in both kernels; 256 (single CTA) or 128 (each
  // CTA of a pair) of B.
  if (!make_operand_map(&ma, L.a, es, L.a_mn_major, p.m, p.k, L.lda, L.stride_a, a_bdim, 128))
    return cudaErrorInvalidValue;
  if (!make_operand_map(&mb, L.b, es, L.b_mn_major, p.n, p.k, L.ldb, L.stride_b, b_bdim, pair ? 128 : tile_n))
    return cudaErrorInvalidValue;
  const long long tiles = (long long)p.m_tiles * p.n_tiles * p.batch;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (p.n_peers > 0) {
    // Replicated output: the 16-bit kinds only (the shard layer's bf16 / fp16 path).
    if (L.kind != kKindF16 || L.out == kOutS32) return cudaErrorNotSupported;
  }
  if (pair) {
    int pairs = (int)(tiles < num_sms / 2 ? tiles : num_sms / 2);
    p.sk_dp_tiles = (int)tiles;
    p.sk_tiles = 0;
    p.sk_splits = 1;
    SkPlan sp;
    // Split-K tail over CTA pairs: the plan of the single-CTA kernel with a
    // pair as the unit of parallelism; each cut unit holds two 128 x 256
    // partial slots (one per CTA).
    if (L.sk_ws && p.n_peers == 0 && plan_splitk(tiles, p.k_blocks, num_sms / 2, sp) &&
        L.sk_ws_bytes >= splitk_bytes(sp, 2)) {
      p.sk_dp_tiles = (int)sp.dp_tiles;
      p.sk_tiles = (int)sp.sk_tiles;
      p.sk_splits = sp.splits;
      p.sk_part = static_cast<uint32_t*>(L.sk_ws);
      p.sk_count = reinterpret_cast<int*>(static_cast<uint8_t*>(L.sk_ws) + (size_t)sp.sk_tiles * sp.splits * 2 *
                                                                             kTileM * kTileN * sizeof(uint32_t));
      const cudaError_t e =
          cudaMemsetAsync(p.sk_count, 0, (size_t)sp.sk_tiles * 2 * kEpiWarps * sizeof(int), stream);
      if (e != cudaSuccess) return e;
      const long long units = sp.dp_tiles + sp.sk_tiles * sp.splits;
      pairs = (int)(units < num_sms / 2 ? units : num_sms / 2);
    }
    const int g2 = 2 * pairs;
    if (p.probe && p.probe_capacity < g2) return cudaErrorInvalidValue;
    if (p.n_peers > 0) {
      switch (L.out) {
        case kOutF32: return launch_pair_impl<kKindF16, kOutF32, true>(ma, mb, p, g2, stream);
        case kOutBF16: return launch_pair_impl<kKindF16, kOutBF16, true>(ma, mb, p, g2, stream);
        case kOutF16: return launch_pair_impl<kKindF16, kOutF16, true>(ma, mb, p, g2, stream);
        default: return cudaErrorNotSupported;
      }
    }
    switch (L.kind * 4 + L.out) {
      case kKindF16 * 4 + kOutF32: return launch_pair_impl<kKindF16, kOutF32>(ma, mb, p, g2, stream);
      case kKindF16 * 4 + kOutBF16: return launch_pair_impl<kKindF16, kOutBF16>(ma, mb, p, g2, stream);
      case kKindF16 * 4 + kOutF16: return launch_pair_impl<kKindF16, kOutF16>(ma, mb, p, g2, stream);
      case kKindI8 * 4 + kOutS32: return launch_pair_impl<kKindI8, kOutS32>(ma, mb, p, g2, stream);
      case kKindI8 * 4 + kOutBF16: return launch_pair_impl<kKindI8, kOutBF16>(ma, mb, p, g2, stream);
      case kKindI8 * 4 + kOutF32: return launch_pair_impl<kKindI8, kOutF32>(ma, mb, p, g2, stream);
      case kKindF8 * 4 + kOutBF16: return launch_pair_impl<kKindF8, kOutBF16>(ma, mb, p, g2, stream);
      case kKindF8 * 4 + kOutF32: return launch_pair_impl<kKindF8, kOutF32>(ma, mb, p, g2, stream);
      default: return cudaErrorNotSupported;
    }
  }
  int grid = (int)(tiles < num_sms ? tiles : num_sms);
  p.sk_dp_tiles = (int)tiles;
  p.sk_tiles = 0;
  p.sk_splits = 1;
  if (splitk) {
    p.sk_dp_tiles = (int)sp.dp_tiles;
    p.sk_tiles = (int)sp.sk_tiles;
    p.sk_splits = sp.splits;
    p.sk_part = static_cast<uint32_t*>(L.sk_ws);
    p.sk_count = reinterpret_cast<int*>(static_cast<uint8_t*>(L.sk_ws) +
                                        (size_t)sp.sk_tiles * sp.splits * kTileM * kTileN * sizeof(uint32_t));
    const cudaError_t e = cudaMemsetAsync(p.sk_count, 0, (size_t)sp.sk_tiles * kEpiWarps * sizeof(int), stream);
    if (e != cudaSuccess) return e;
    const long long units = sp.dp_tiles + sp.sk_tiles * sp.splits;
    grid = (int)(units < num_sms ? units : num_sms);
  }
  if (p.probe && p.probe_capacity < grid) return cudaErrorInvalidValue;
  if (p.n_peers > 0) {
    switch (L.out) {
      case kOutF32: return launch_impl<kKindF16, kOutF32, false, true>(ma, mb, p, grid, stream);
      case kOutBF16: return launch_impl<kKindF16, kOutBF16, false, true>(ma, mb, p, grid, stream);
      case kOutF16: return launch_impl<kKindF16, kOutF16, false, true>(ma, mb, p, grid, stream);
      default: return cudaErrorNotSupported;
    }
  }
  switch (L.kind * 4 + L.out) {
    case kKindF16 * 4 + kOutF32: return launch_impl<kKindF16, kOutF32>(ma, mb, p, grid, stream);
    case kKindF16 * 4 + kOutBF16: return launch_impl<kKindF16, kOutBF16>(ma, mb, p, grid, stream);
    case kKindF16 * 4 + kOutF16: return launch_impl<kKindF16, kOutF16>(ma, mb, p, grid, stream);
    case kKindI8 * 4 + kOutS32: return launch_impl<kKindI8, kOutS32>(ma, mb, p, grid, stream);
    case kKindI8 * 4 + kOutBF16: return launch_impl<kKindI8, kOutBF16>(ma, mb, p, grid, stream);
    case kKindI8 * 4 + kOutF32: return launch_impl<kKindI8, kOutF32>(ma, mb, p, grid, stream);
    case kKindF8 * 4 + kOutBF16: return launch_impl<kKindF8, kOutBF16>(ma, mb, p, grid, stream);
    case kKindF8 * 4 + kOutF32: return launch_impl<kKindF8, kOutF32>(ma, mb, p, grid, stream);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace grx
