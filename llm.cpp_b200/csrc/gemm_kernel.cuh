// tcgen05 GEMM kernel templates (sm_100a), shared by the translation units
// that instantiate them: gemm_{bf16,tf32}_{pair256,pair128,cta}.cu compile the
// kernels of one operand type and tile shape each (in parallel), gemm.cu holds
// the planner, the split-K reduction and the C entry points.
//
// tcgen05 GEMM for sm_100a: D[M,N] = epilogue(A[M,K] * B[N,K]^T).
//
// One persistent, warp-specialised kernel serves the three contractions of a
// GPT-2 linear layer (reference gpt2/cuda/matmul.cu:223-449):
//   forward  out  = inp * W^T      A = inp  (K-major),  B = W    (K-major)
//   dinp     dinp = dout * W       A = dout (K-major),  B = W    (N-major)
//   dweight  dW   = dout^T * inp   A = dout (M-major),  B = inp  (N-major)
// Operand majorness is a template parameter; the smem descriptors and the
// instruction descriptor's transpose bits absorb it, so no operand is ever
// transposed in memory.
//
// CTA pairs (kPair): a cluster of two CTAs on two SMs computes a 256 x BN
// tile with cta_group::2 MMAs issued by the leader CTA. Each CTA stages its
// own 128 rows of A and half of the BN rows of B, so per SM the operand
// traffic per MMA FLOP is a third lower than with one CTA per tile; each CTA's
// TMEM holds its 128 x BN slice of the accumulator. Without kPair one CTA
// computes a 128 x BN tile alone (small M).
//
// CTA = 10 warps: warp 0 issues TMA loads into a kStages-deep ring of 128B-
// swizzled smem stages, warp 1 owns TMEM and (in the leader) issues
// tcgen05.mma from one thread, warps 2..9 drain the double-buffered TMEM
// accumulator (two warps per 32-lane TMEM quarter, one per column half)
// through the fused epilogue (bias, residual add, GELU, GELU-backward,
// accumulate) while the next tile's mainloop runs. Split-K writes fp32
// partial tiles to a caller workspace, reduced deterministically by
// gemm_splitk_reduce.
#pragma once
#include <algorithm>
#include <cstdio>

#include "ptx.cuh"
#include "runtime.h"

namespace llmk {

struct EpiParams {
  void* D;
  long long ldd;
  int d_bf16;
  const float* bias;
  const float* residual;
  long long ldr;
  __nv_bfloat16* aux;
  long long ldaux;
  int flags;
  float* partial;  // split-K: fp32 [splits][M][N] workspace (raw accumulators)
  int aux_tma;     // GELU pre-activation leaves by TMA store (aux dtype == D dtype)
  int op;          // kOp*: the epilogue program the drain runs
  // Row softmax statistics of D as stored (bf16-rounded for a bf16 D): for
  // each row and each 64-column slot, (max, sum exp(x - max)) over the slot's
  // columns below stats_cols, at stats[slot * M + row].
  float2* stats;
  int stats_cols;
};

// Epilogue programs. The drain of a chunk runs straight-line code for the
// operations the GEMM actually has: a generic program that tests every flag
// for every 8-column group branches over most of its code, and on B200 the
// instruction fetches of that sparse path cost more than the work itself
// (about 1.3 us per 4 KB chunk with nothing to apply). The common programs
// are therefore compiled separately; kOpGeneric keeps the flag-driven path
// for every other combination.
//   kOpNone      store the accumulator (also split-K partial tiles)
//   kOpBias      + bias
//   kOpBiasRes   + bias + fp32 residual, fp32 D (the residual-stream GEMMs);
//                the residual arrives by TMA loads (epilogue_operand_role)
//   kOpBiasGelu  + bias, GELU, pre-activation by TMA store (aux type == D type)
//   kOpGeluBwd   * GELU'(pre-activation), aux type == D type, loaded by TMA
//   kOpStats     + bias, and the rows' softmax statistics (the logits GEMM)
// Each is a kernel template argument: one kernel holds one program.
enum : int { kOpNone = 0, kOpBias = 1, kOpBiasRes = 2, kOpBiasGelu = 3, kOpGeluBwd = 4, kOpGeneric = 5, kOpStats = 6 };

// One launcher per operand type and tile shape (kind 0 = single CTA, BN 128;
// 1 = CTA pair, BN 128; 2 = CTA pair, BN 256), each in its own unit.
#define LLMK_GEMM_DISPATCH_DECL(name)                                                                           \
  int name(int a_trans, int b_trans, const void* A, long long lda, const void* B, long long ldb, int M, int N, \
           int K, const EpiParams& ep, int splits, cudaStream_t s)
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_bf16_pair256);
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_bf16_pair128);
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_bf16_cta);
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_tf32_pair256);
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_tf32_pair128);
LLMK_GEMM_DISPATCH_DECL(gemm_dispatch_tf32_cta);

namespace {


// Staging buffers per epilogue warp: two (alternating TMA-store buffers), or
// three for the programs whose drain reads a per-element operand of D's shape
// (it arrives by TMA loads into the buffers, two chunks ahead of the drain).
constexpr int op_bufs(int op) { return (op == kOpBiasRes || op == kOpGeluBwd) ? 3 : 2; }

template <bool kTF32, bool kAMN, bool kBMN, int kBN, bool kPair, int kBufs = 2>
struct Cfg {
  static constexpr int kElem = kTF32 ? 4 : 2;
  static constexpr int BM = 128;                   // accumulator rows per CTA
  static constexpr int kMmaM = kPair ? 256 : 128;  // rows per tile (per MMA)
  static constexpr int BNC = kPair ? kBN / 2 : kBN;  // B rows this CTA stages
  static constexpr int BK = 128 / kElem;           // K per stage (one 128-byte swizzle row)
  static constexpr int kAtomMN = 128 / kElem;      // M/N elements per 128-byte atom (MN-major)
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BNC * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int kRowsPerMma = 32 / kElem;   // K of one MMA (16 bf16, 8 tf32)
  static constexpr int kKSteps = BK / kRowsPerMma; // 4
  static constexpr int kTmemCols = 2 * kBN;        // two accumulators
  // MN-major operands: tf32 needs the 32-byte-atom 128B swizzle (4-row
  // groups, 512 B apart); bf16 the plain 128B swizzle (8-row groups, 1024 B).
  static constexpr uint32_t kMNLayout = kTF32 ? kLayoutSW128Base32 : kLayoutSW128;
  static constexpr uint32_t kMNSbo = kTF32 ? 512 : 1024;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  // Epilogue staging for TMA stores: 8 warps x kBufs buffers x [32 rows x 128 B].
  static constexpr int STAGING_BYTES = kEpiWarps * kBufs * 4096;
  // barriers: the pipeline's at BAR_OFF, the operand loads' at BAR_OFF + 256
  static constexpr int kBarBytes = 512;
  // as many operand stages as fit beside the staging buffers (227 KB per CTA)
  static constexpr int kStagesFit = (232448 - 1024 - kBarBytes - STAGING_BYTES) / STAGE_BYTES;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int STAGING_OFF = kStages * STAGE_BYTES;
  static constexpr int BAR_OFF = STAGING_OFF + STAGING_BYTES;
  static constexpr size_t SMEM = size_t(BAR_OFF) + kBarBytes + 1024;
  static_assert(kBN == 128 || kBN == 256, "BN");
  static_assert(kStages >= 3, "stages");
  static_assert(kBufs == 2 || kBufs == 3, "staging buffers");
  static_assert(8 * (2 * 8 + 5) + 8 <= 256 && 256 + 8 * kEpiWarps * 3 <= kBarBytes, "barrier area");
  static_assert(!kBMN || BNC % kAtomMN == 0, "B atoms");
};

// Tile order: groups of G m-blocks; inside a group m runs fastest, so the
// CTAs in flight share B panels, and the group's G A panels stay in L2 while
// the group walks every n-block. G = num_m (one group) reads B from DRAM once
// and sweeps A from L2: the host picks it when B is the operand that does not
// fit in L2 beside the output stream (the tied lm_head forward).
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int G, int& m_blk, int& n_blk, int& split) {
  const int per_split = num_m * num_n;
  split = t / per_split;
  t -= split * per_split;
  const int per_group = G * num_n;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int m_first = g * G;
  const int gs = min(G, num_m - m_first);
  m_blk = m_first + r % gs;
  n_blk = r / gs;
}

__device__ __forceinline__ void load8(const float* p, float* v) {
  float4 a = reinterpret_cast<const float4*>(p)[0];
  float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(float* p, const float* v) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Epilogue operations on 8 consecutive columns [gn, gn+8) of row gm (all in
// bounds) except the final store, in two parts: epi_pre8 adds bias and
// residual (giving the GELU pre-activation); epi_post8 stores the
// pre-activation when asked (store_aux), applies GELU / GELU-backward and
// accumulates onto the old D. A bf16 output takes the SFU tanh in the GELU
// pair (its error is below the bf16 rounding).
__device__ __forceinline__ void epi_pre8(const EpiParams& ep, long long gm, int gn, float* v) {
  float t[8];
  if (ep.bias) {
    load8(ep.bias + gn, t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] += t[j];
  }
  if (ep.residual) {
    load8(ep.residual + gm * ep.ldr + gn, t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] += t[j];
  }
}
__device__ __forceinline__ void epi_post8(const EpiParams& ep, long long gm, int gn, float* v, bool store_aux) {
  float t[8];
  if (ep.flags & LLMK_EPI_GELU) {
    if (ep.aux && store_aux) {
      if (ep.flags & LLMK_EPI_AUX_F32) store8(reinterpret_cast<float*>(ep.aux) + gm * ep.ldaux + gn, v);
      else store8_bf16(ep.aux + gm * ep.ldaux + gn, v);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = ep.d_bf16 ? gelu_tanh_fast(v[j]) : gelu_tanh(v[j]);
  } else if (ep.flags & LLMK_EPI_GELU_BWD) {
    if (ep.flags & LLMK_EPI_AUX_F32) load8(reinterpret_cast<const float*>(ep.aux) + gm * ep.ldaux + gn, t);
    else load8_bf16(ep.aux + gm * ep.ldaux + gn, t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= ep.d_bf16 ? gelu_tanh_grad_fast(t[j]) : gelu_tanh_grad(t[j]);
  }
  if (ep.flags & LLMK_EPI_ACCUMULATE) {
    if (ep.d_bf16) load8_bf16(static_cast<const __nv_bfloat16*>(ep.D) + gm * ep.ldd + gn, t);
    else load8(static_cast<const float*>(ep.D) + gm * ep.ldd + gn, t);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] += t[j];
  }
}


// Columns [8k, 8k + 8) of a chunk row held as eight 16-byte pieces (bf16: one
// piece per group; fp32: two), as floats.
template <bool kBF16>
__device__ __forceinline__ void chunk_unpack8(const uint4* pre, int k, float* t) {
  if constexpr (kBF16) {
    const uint4 u = pre[k];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      t[2 * i] = __uint_as_float(w[i] << 16);
      t[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    const uint4 a = pre[2 * k], b = pre[2 * k + 1];
    t[0] = __uint_as_float(a.x); t[1] = __uint_as_float(a.y); t[2] = __uint_as_float(a.z); t[3] = __uint_as_float(a.w);
    t[4] = __uint_as_float(b.x); t[5] = __uint_as_float(b.y); t[6] = __uint_as_float(b.z); t[7] = __uint_as_float(b.w);
  }
}

// Writes the 8 values of column group k (8 columns) of this lane's row into a
// 128B-swizzled [32 rows x 128 B] staging buffer: bf16 = one 16-byte chunk,
// fp32 = two.
template <bool kBF16>
__device__ __forceinline__ void stage8(uint8_t* buf, int lane, int k, const float* v) {
  const int r7 = lane & 7;
  if constexpr (kBF16) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(buf + lane * 128 + ((k ^ r7) << 4)) = u;
  } else {
    *reinterpret_cast<uint4*>(buf + lane * 128 + (((2 * k) ^ r7) << 4)) =
        make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
    *reinterpret_cast<uint4*>(buf + lane * 128 + (((2 * k + 1) ^ r7) << 4)) =
        make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]), __float_as_uint(v[7]));
  }
}


// Folds columns [gn0, gn0 + CW) of this lane's row into the running softmax
// statistics (m, s) and writes them out at the end of each 64-column slot.
// For a bf16 D the values are first rounded as the store will round them, so
// the statistics describe the stored logits exactly.
template <bool kBF16, int CW>
__device__ __forceinline__ void rowstats_chunk(const EpiParams& ep, long long gm, int gn0, int N, int M, float* v,
                                               float& m, float& s) {
  if constexpr (kBF16) {
#pragma unroll
    for (int j = 0; j < CW; j += 2) {
      const uint32_t u = pack_bf16x2(v[j], v[j + 1]);
      v[j] = __uint_as_float(u << 16);
      v[j + 1] = __uint_as_float(u & 0xffff0000u);
    }
  }
  // columns at or past stats_cols only in the chunk that holds the vocabulary end
  const bool full = gn0 + CW <= ep.stats_cols;
  float cm = -INFINITY;
#pragma unroll
  for (int j = 0; j < CW; ++j)
    if (full || gn0 + j < ep.stats_cols) cm = fmaxf(cm, v[j]);
  if (cm > -INFINITY) {
    const float mn = fmaxf(m, cm);
    const float m2 = mn * kLog2e;
    float acc = s * ex2_approx(m * kLog2e - m2);
#pragma unroll
    for (int j = 0; j < CW; ++j)
      if (full || gn0 + j < ep.stats_cols) acc += ex2_approx(fmaf(v[j], kLog2e, -m2));
    m = mn;
    s = acc;
  }
  if (((gn0 + CW) & 63) == 0 || gn0 + CW >= N) {
    if (gm < M) ep.stats[static_cast<long long>(gn0 >> 6) * M + gm] = make_float2(m, s);
    m = -INFINITY;
    s = 0.f;
  }
}

// Drains columns [c_begin, c_end) of one warp's 32 accumulator rows (TMEM
// lanes from `tsrc`) through epilogue program kOp in chunks of 4 KB: 64 bf16
// or 32 fp32 columns. Each chunk is written 128B-swizzled into one of the
// warp's two staging buffers and stored by one lane with a TMA store; the
// buffers alternate, so a chunk's smem writes only wait for the store issued
// two chunks earlier. kAux: the GELU pre-activation is staged too and leaves
// by a second TMA store (tmX); kOpBiasGelu stores it (first buffer) before
// computing the GELU and D (second buffer) after, so each buffer waits only
// for its own previous store. Rows / columns past M / N are clipped by the
// tensor maps. kStats: row softmax statistics as well (bias only, no split-K).
template <bool kBF16, bool kAux, int kOp, bool kStats = false>
__device__ __forceinline__ void epilogue_cols(const EpiParams& ep, const CUtensorMap* tmD, const CUtensorMap* tmX,
                                              uint32_t tsrc, int row0, int n0, int c_begin, int c_end, int sp, int M,
                                              int N, int lane, uint8_t* stg, uint32_t& nstore) {
  constexpr int CW = kBF16 ? 64 : 32;  // columns per chunk
  static_assert(op_bufs(kOp) == 2, "operand-loading programs drain in epilogue_operand_role");
  const long long gm = row0 + lane;
  const bool row_ok = gm < M && !ep.partial;
  float st_m = -INFINITY, st_s = 0.f;
#pragma unroll 1
  for (int c0 = c_begin; c0 < c_end; c0 += CW) {
    const int gn0 = n0 + c0;
    if (gn0 >= N) break;
    float v[CW];
    {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tsrc + c0, r);
      if constexpr (kBF16) {
        uint32_t r2[32];
        tmem_ld_32x32b_x32(tsrc + c0 + 32, r2);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[32 + j] = __uint_as_float(r2[j]);
      } else {
        tmem_ld_wait();
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    }
    uint8_t* buf = kAux ? stg + 4096 : stg + (nstore & 1u) * 4096;
    if constexpr (kStats) {
      if (ep.bias) {
#pragma unroll
        for (int k = 0; k < CW / 8; ++k)
          if (gn0 + k * 8 < N) epi_pre8(ep, gm, gn0 + k * 8, v + k * 8);
      }
      rowstats_chunk<kBF16, CW>(ep, gm, gn0, N, M, v, st_m, st_s);
    } else if constexpr (kOp == kOpGeneric) {
      if constexpr (kAux) {
        // both buffers: every earlier store must be done reading
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
      }
      if (row_ok) {
#pragma unroll
        for (int k = 0; k < CW / 8; ++k) {
          if (gn0 + k * 8 < N) {
            epi_pre8(ep, gm, gn0 + k * 8, v + k * 8);
            if constexpr (kAux) stage8<kBF16>(stg, lane, k, v + k * 8);
            epi_post8(ep, gm, gn0 + k * 8, v + k * 8, !kAux);
          }
        }
      }
    } else if constexpr (kOp != kOpNone) {
      if (row_ok) {
        // column clamped into [0, N): no branch per group
        float t[8];
#pragma unroll
        for (int k = 0; k < CW / 8; ++k) {
          const int gc = gn0 + k * 8 < N ? gn0 + k * 8 : N - 8;
          if constexpr (kOp == kOpBias || kOp == kOpBiasGelu) {
            load8(ep.bias + gc, t);
#pragma unroll
            for (int j = 0; j < 8; j += 2)
              f2_unpack(f2_add(f2_pack(v[k * 8 + j], v[k * 8 + j + 1]), f2_pack(t[j], t[j + 1])), v[k * 8 + j],
                        v[k * 8 + j + 1]);
          }
        }
      }
      if constexpr (kOp == kOpBiasGelu) {
        // the pre-activation: first buffer, free once its previous store has
        // read it (the newest group, the previous D store, may still be reading)
        if (lane == 0) bulk_wait_read1();
        __syncwarp();
#pragma unroll
        for (int k = 0; k < CW / 8; ++k) stage8<kBF16>(stg, lane, k, v + k * 8);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmX, stg, gn0, row0);
          bulk_commit();
        }
        if constexpr (kBF16) {
#pragma unroll
          for (int j = 0; j < CW; j += 2) f2_unpack(gelu_tanh_fast2(f2_pack(v[j], v[j + 1])), v[j], v[j + 1]);
        } else {
#pragma unroll
          for (int j = 0; j < CW; ++j) v[j] = gelu_tanh(v[j]);
        }
      }
    }
    if constexpr (!kAux || kOp == kOpBiasGelu) {
      // the store that last read this buffer must be done reading (the
      // newest group, a store from the other buffer, may still be reading)
      if (lane == 0) bulk_wait_read1();
      __syncwarp();
    }
#pragma unroll
    for (int k = 0; k < CW / 8; ++k) stage8<kBF16>(buf, lane, k, v + k * 8);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (ep.partial) tma_store_3d(tmD, buf, gn0, row0, sp);
      else tma_store_2d(tmD, buf, gn0, row0);
      if constexpr (kAux && kOp != kOpBiasGelu) tma_store_2d(tmX, stg, gn0, row0);
      bulk_commit();
    }
    ++nstore;
  }
}

// What the epilogue role of one warp needs to walk its tiles.
struct EpiRole {
  int unit, units, num_tiles, num_m, num_n, group_m;
  int rank_rows;  // this CTA's first accumulator row inside a tile (rank * 128)
  int q, half, lane, M, N;
  uint32_t tmem_base;
  unsigned int* status;
  volatile int* abort_flag;
};

// Epilogue role of the programs whose drain reads a per-element operand of D's
// shape: kOpBiasRes (D = acc + bias + residual, fp32) and kOpGeluBwd (D = acc *
// GELU'(pre-activation), the pre-activation in D's type). The operand arrives
// by TMA tile loads (box = one 4 KB chunk, 128B-swizzled exactly as the D chunk
// is staged) into the warp's three staging buffers: chunk n's operand lands in
// buffer n % 3, each lane reads its row from there (conflict-free: the swizzle
// spreads a quarter-warp's 16-byte pieces over all banks), writes its result
// over it, and one lane TMA-stores the buffer. Loads run two chunks ahead of
// the drain and across tile boundaries: the load of chunk n + 2 goes into the
// buffer of chunk n - 1 as soon as that chunk's store has finished reading it,
// so the operand waits in shared memory when the accumulator is ready.
// Rows / columns past M / N load as zeros and are clipped by D's tensor map.
// tmX maps the operand with D's chunk box.
template <bool kBF16, int kOp, int kBN, int kMmaM, bool kPair>
__device__ __forceinline__ void epilogue_operand_role(const EpiParams& ep, const CUtensorMap* tmD,
                                                      const CUtensorMap* tmX, const EpiRole& r, uint64_t* accf,
                                                      uint64_t* acce, uint32_t acce_leader0, uint64_t* opbar,
                                                      uint8_t* stg) {
  constexpr int CW = kBF16 ? 64 : 32;  // columns per 4 KB chunk
  const int lane = r.lane;
  const int cb = r.half * (kBN / 2), ce = cb + kBN / 2;
  // The load sequence (lane 0 only): tile lt, column lc of the next chunk to load.
  int lt = r.unit, lc = cb;
  uint32_t nload = 0;
  auto issue = [&]() {
    while (lt < r.num_tiles) {
      int mb, nb, sp;
      tile_coords(lt, r.num_m, r.num_n, r.group_m, mb, nb, sp);
      if (lc < ce && nb * kBN + lc < r.N) {
        const int j = static_cast<int>(nload % 3u);
        mbar_arrive_expect_tx(opbar + j, 4096);
        tma_load_2d(stg + j * 4096, tmX, opbar + j, nb * kBN + lc, mb * kMmaM + r.rank_rows + r.q * 32);
        ++nload;
        lc += CW;
        return;
      }
      lt += r.units;
      lc = cb;
    }
  };
  if (lane == 0) {
    issue();
    issue();
  }
  uint32_t n = 0;  // chunks drained (= stores issued) by this warp
  bool failed = false;
  int local = 0;
  for (int tile = r.unit; tile < r.num_tiles && !failed; tile += r.units, ++local) {
    int mb, nb, sp;
    tile_coords(tile, r.num_m, r.num_n, r.group_m, mb, nb, sp);
    const int row0 = mb * kMmaM + r.rank_rows + r.q * 32;
    const int n0 = nb * kBN;
    const int acc = local & 1;
    const uint32_t aphase = (local >> 1) & 1;
    {
      // while the tile's MMAs run, pull this lane's row segment of the operand
      // into L2 (the chunk loads then find it there)
      const long long gm = row0 + lane;
      const int c0 = n0 + cb;
      if (gm < r.M && c0 < r.N) {
        const uint32_t ncol = static_cast<uint32_t>(min(kBN / 2, r.N - c0));
        if constexpr (kOp == kOpBiasRes) prefetch_l2_bulk(ep.residual + gm * ep.ldr + c0, ncol * 4);
        else prefetch_l2_bulk(reinterpret_cast<const uint8_t*>(ep.aux) + (gm * ep.ldaux + c0) * (kBF16 ? 2 : 4),
                              ncol * (kBF16 ? 2 : 4));
      }
    }
    bool ok = mbar_wait(accf + acc, aphase, r.status, r.abort_flag);
    if (!__all_sync(0xffffffffu, ok)) { failed = true; break; }
    tc_fence_after();
    const uint32_t tsrc = r.tmem_base + (static_cast<uint32_t>(r.q * 32) << 16) + acc * kBN;
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += CW) {
      const int gn0 = n0 + c0;
      if (gn0 >= r.N) break;
      float v[CW];
      {
        uint32_t t32[32];
        tmem_ld_32x32b_x32(tsrc + c0, t32);
        if constexpr (kBF16) {
          uint32_t t32b[32];
          tmem_ld_32x32b_x32(tsrc + c0 + 32, t32b);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[32 + j] = __uint_as_float(t32b[j]);
        } else {
          tmem_ld_wait();
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(t32[j]);
      }
      const int b = static_cast<int>(n % 3u);
      uint8_t* buf = stg + b * 4096;
      ok = mbar_wait(opbar + b, (n / 3u) & 1u, r.status, r.abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { failed = true; break; }
      const int r7 = lane & 7;
      uint4 pre[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pre[j] = *reinterpret_cast<const uint4*>(buf + lane * 128 + ((j ^ r7) << 4));
      float t[8];
#pragma unroll
      for (int k = 0; k < CW / 8; ++k) {
        chunk_unpack8<kBF16>(pre, k, t);
        if constexpr (kOp == kOpBiasRes) {
          // column clamped into [0, N): no branch per group
          const int gc = gn0 + k * 8 < r.N ? gn0 + k * 8 : r.N - 8;
          float bb[8];
          load8(ep.bias + gc, bb);
#pragma unroll
          for (int j = 0; j < 8; j += 2) {  // (acc + bias) + residual
            const uint64_t r = f2_add(f2_add(f2_pack(v[k * 8 + j], v[k * 8 + j + 1]), f2_pack(bb[j], bb[j + 1])),
                                      f2_pack(t[j], t[j + 1]));
            f2_unpack(r, v[k * 8 + j], v[k * 8 + j + 1]);
          }
        } else {
          if constexpr (kBF16) {
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const uint64_t g = f2_mul(f2_pack(v[k * 8 + j], v[k * 8 + j + 1]), gelu_tanh_grad_fast2(f2_pack(t[j], t[j + 1])));
              f2_unpack(g, v[k * 8 + j], v[k * 8 + j + 1]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[k * 8 + j] *= gelu_tanh_grad(t[j]);
          }
        }
      }
      // chunk n - 1's store has read buffer (n + 2) % 3: load chunk n + 2 into it
      if (lane == 0) {
        bulk_wait_read0();
        issue();
      }
      // the result goes over the operand, each lane on its own row
#pragma unroll
      for (int k = 0; k < CW / 8; ++k) stage8<kBF16>(buf, lane, k, v + k * 8);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmD, buf, gn0, row0);
        bulk_commit();
      }
      ++n;
    }
    if (failed) break;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (kPair) mbar_arrive_cluster(acce_leader0 + acc * 8);
      else mbar_arrive(acce + acc);
    }
  }
  // after a failed wait: let the loads still in flight land before the CTA exits
  if (lane == 0) {
    for (uint32_t i = n; i < nload; ++i) mbar_wait(opbar + i % 3u, (i / 3u) & 1u, nullptr, nullptr);
  }
  __syncwarp();
}

template <bool kTF32, bool kAMN, bool kBMN, int kBN, bool kPair, int kOp>
__global__ void __launch_bounds__(Cfg<kTF32, kAMN, kBMN, kBN, kPair>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmX, EpiParams ep,
                   int M, int N, int K, int splits, int group_m, unsigned int* status) {
  using C = Cfg<kTF32, kAMN, kBMN, kBN, kPair, op_bufs(kOp)>;
  constexpr bool kOperandLoads = op_bufs(kOp) == 3;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::kStages;
  uint64_t* accf = empty + C::kStages;
  uint64_t* acce = accf + 2;
  uint64_t* done = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* opbar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF + 256);  // 3 per epilogue warp

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf + a, 1);
      // one arrival per epilogue warp, of both CTAs of a pair (on the leader's barrier)
      mbar_init(acce + a, kPair ? 2 * C::kEpiWarps : C::kEpiWarps);
    }
    mbar_init(done, 1);
    if constexpr (kOperandLoads) {
      for (int i = 0; i < 3 * C::kEpiWarps; ++i) mbar_init(opbar + i, 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if (kPair) {
      tmem_alloc_pair(tmem_slot, C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncwarp();
  // the peer's barriers are initialised before any remote arrive / complete_tx
  if (kPair) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + C::kMmaM - 1) / C::kMmaM;
  const int num_n = (N + kBN - 1) / kBN;
  const int num_tiles = num_m * num_n * splits;
  const int num_kb = (K + C::BK - 1) / C::BK;
  const int kb_per = (num_kb + splits - 1) / splits;
  const int unit = kPair ? static_cast<int>(blockIdx.x) >> 1 : static_cast<int>(blockIdx.x);
  const int units = kPair ? static_cast<int>(gridDim.x) >> 1 : static_cast<int>(gridDim.x);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = unit; tile < num_tiles; tile += units) {
        int mb, nb, sp;
        tile_coords(tile, num_m, num_n, group_m, mb, nb, sp);
        const int m0 = mb * C::kMmaM + static_cast<int>(rank) * C::BM;
        const int nc0 = nb * kBN + static_cast<int>(rank) * C::BNC;
        const int kb0 = sp * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1u, status, abort_flag)) { ok = false; break; }
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          const int k0 = kb * C::BK;
          if (kPair) {
            // both CTAs' loads complete on the leader's full barrier, which
            // expects the bytes of the pair
            const uint32_t fb = mapa_shared(smem_u32(full + stage), 0);
            if (leader) mbar_arrive_expect_tx(full + stage, 2 * C::STAGE_BYTES);
            if (!kAMN) {
              tma_load_2d_pair(sA, &tmA, fb, k0, m0);
            } else {
#pragma unroll
              for (int j = 0; j < C::BM / C::kAtomMN; ++j)
                tma_load_2d_pair(sA + j * C::BK * 128, &tmA, fb, m0 + j * C::kAtomMN, k0);
            }
            if (!kBMN) {
              tma_load_2d_pair(sB, &tmB, fb, k0, nc0);
            } else {
#pragma unroll
              for (int j = 0; j < C::BNC / C::kAtomMN; ++j)
                tma_load_2d_pair(sB + j * C::BK * 128, &tmB, fb, nc0 + j * C::kAtomMN, k0);
            }
          } else {
            mbar_arrive_expect_tx(full + stage, C::STAGE_BYTES);
            if (!kAMN) {
              tma_load_2d(sA, &tmA, full + stage, k0, m0);
            } else {
#pragma unroll
              for (int j = 0; j < C::BM / C::kAtomMN; ++j)
                tma_load_2d(sA + j * C::BK * 128, &tmA, full + stage, m0 + j * C::kAtomMN, k0);
            }
            if (!kBMN) {
              tma_load_2d(sB, &tmB, full + stage, k0, nc0);
            } else {
#pragma unroll
              for (int j = 0; j < C::BNC / C::kAtomMN; ++j)
                tma_load_2d(sB + j * C::BK * 128, &tmB, full + stage, nc0 + j * C::kAtomMN, k0);
            }
          }
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = idesc_f32acc(C::kMmaM, kBN, kTF32 ? kFmtTF32 : kFmtBF16, kAMN, kBMN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = unit; tile < num_tiles && ok; tile += units, ++local) {
        int mb, nb, sp;
        tile_coords(tile, num_m, num_n, group_m, mb, nb, sp);
        const int kb0 = sp * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!mbar_wait(acce + acc, aphase ^ 1u, status, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full + stage, phase, status, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sA = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sB = sA + C::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < C::kKSteps; ++ks) {
            uint64_t adesc, bdesc;
            if (!kAMN) adesc = sdesc_sw128(sA + ks * 32, 16, 1024);
            else adesc = sdesc_sw128(sA + ks * C::kRowsPerMma * 128, C::BK * 128, C::kMNSbo, C::kMNLayout);
            if (!kBMN) bdesc = sdesc_sw128(sB + ks * 32, 16, 1024);
            else bdesc = sdesc_sw128(sB + ks * C::kRowsPerMma * 128, C::BK * 128, C::kMNSbo, C::kMNLayout);
            const uint32_t accum = (kb > kb0 || ks > 0) ? 1u : 0u;
            if (kPair) {
              if (kTF32) mma_tf32_ss_pair(d_tmem, adesc, bdesc, idesc, accum);
              else mma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, accum);
            } else {
              if (kTF32) mma_tf32_ss(d_tmem, adesc, bdesc, idesc, accum);
              else mma_f16_ss(d_tmem, adesc, bdesc, idesc, accum);
            }
          }
          // the stage is free in both CTAs once these MMAs have read it
          if (kPair) mma_commit_pair(empty + stage, 3);
          else mma_commit(empty + stage);
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if (kPair) mma_commit_pair(accf + acc, 3);
        else mma_commit(accf + acc);
      }
      // All MMAs issued by this thread complete before TMEM is released.
      if (kPair) mma_commit_pair(done, 1);
      else mma_commit(done);
      mbar_wait(done, 0, status, nullptr);
    }
    __syncwarp();
  } else if constexpr (kOperandLoads) {
    const int ew = warp - 2;
    EpiRole r;
    r.unit = unit; r.units = units; r.num_tiles = num_tiles; r.num_m = num_m; r.num_n = num_n; r.group_m = group_m;
    r.rank_rows = static_cast<int>(rank) * C::BM;
    r.q = warp & 3; r.half = ew >> 2; r.lane = lane; r.M = M; r.N = N;
    r.tmem_base = tmem_base; r.status = status; r.abort_flag = abort_flag;
    const uint32_t acce_leader0 = kPair ? mapa_shared(smem_u32(acce), 0) : smem_u32(acce);
    uint8_t* stg = smem + C::STAGING_OFF + ew * (3 * 4096);
    if (kOp == kOpGeluBwd && ep.d_bf16)
      epilogue_operand_role<true, kOp, kBN, C::kMmaM, kPair>(ep, &tmD, &tmX, r, accf, acce, acce_leader0,
                                                             opbar + 3 * ew, stg);
    else
      epilogue_operand_role<false, kOp, kBN, C::kMmaM, kPair>(ep, &tmD, &tmX, r, accf, acce, acce_leader0,
                                                              opbar + 3 * ew, stg);
  } else {
    const int ew = warp - 2;               // epilogue warp 0..7
    const int q = warp & 3;                // TMEM lane quarter this warp may access
    const int half = ew >> 2;              // column half of the tile
    uint8_t* stg = smem + C::STAGING_OFF + ew * 8192;  // two 4 KB buffers, used alternately
    uint32_t nstore = 0;                               // store groups this warp committed
    const uint32_t acce_leader0 = kPair ? mapa_shared(smem_u32(acce), 0) : smem_u32(acce);
    int local = 0;
    for (int tile = unit; tile < num_tiles; tile += units, ++local) {
      int mb, nb, sp;
      tile_coords(tile, num_m, num_n, group_m, mb, nb, sp);
      const int m0 = mb * C::kMmaM + static_cast<int>(rank) * C::BM;
      const int n0 = nb * kBN;
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      const int cb = half * (kBN / 2), ce = cb + kBN / 2;
      {
        // while the tile's MMAs run, pull this thread's row segment of the
        // epilogue's global operands (residual, GELU pre-activation, old D)
        // into L2, so the epilogue's loads do not wait on DRAM
        const long long gm = m0 + q * 32 + lane;
        const int c0 = n0 + cb;
        if (gm < M && c0 < N && !ep.partial) {
          const uint32_t ncol = static_cast<uint32_t>(min(kBN / 2, N - c0));
          if (ep.residual) prefetch_l2_bulk(ep.residual + gm * ep.ldr + c0, ncol * 4);
          if (ep.flags & LLMK_EPI_GELU_BWD) {
            if (ep.flags & LLMK_EPI_AUX_F32)
              prefetch_l2_bulk(reinterpret_cast<const float*>(ep.aux) + gm * ep.ldaux + c0, ncol * 4);
            else
              prefetch_l2_bulk(ep.aux + gm * ep.ldaux + c0, ncol * 2);
          }
          if (ep.flags & LLMK_EPI_ACCUMULATE) {
            if (ep.d_bf16) prefetch_l2_bulk(static_cast<const __nv_bfloat16*>(ep.D) + gm * ep.ldd + c0, ncol * 2);
            else prefetch_l2_bulk(static_cast<const float*>(ep.D) + gm * ep.ldd + c0, ncol * 4);
          }
        }
      }
      bool ok = mbar_wait(accf + acc, aphase, status, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t tsrc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kBN;
      const int r0 = m0 + q * 32;
#define LLMK_EPI_ARGS ep, &tmD, &tmX, tsrc, r0, n0, cb, ce, sp, M, N, lane, stg, nstore
      if constexpr (kOp == kOpStats) {
        if (ep.d_bf16) epilogue_cols<true, false, kOpBias, true>(LLMK_EPI_ARGS);
        else epilogue_cols<false, false, kOpBias, true>(LLMK_EPI_ARGS);
      } else if constexpr (kOp == kOpGeneric) {
        if (ep.d_bf16 && !ep.partial) {
          if (ep.aux_tma) epilogue_cols<true, true, kOpGeneric>(LLMK_EPI_ARGS);
          else epilogue_cols<true, false, kOpGeneric>(LLMK_EPI_ARGS);
        } else {
          if (ep.aux_tma) epilogue_cols<false, true, kOpGeneric>(LLMK_EPI_ARGS);
          else epilogue_cols<false, false, kOpGeneric>(LLMK_EPI_ARGS);
        }
      } else if constexpr (kOp == kOpBiasGelu) {
        if (ep.d_bf16) epilogue_cols<true, true, kOpBiasGelu>(LLMK_EPI_ARGS);
        else epilogue_cols<false, true, kOpBiasGelu>(LLMK_EPI_ARGS);
      } else {
        if (ep.d_bf16 && !ep.partial) epilogue_cols<true, false, kOp>(LLMK_EPI_ARGS);
        else epilogue_cols<false, false, kOp>(LLMK_EPI_ARGS);
      }
#undef LLMK_EPI_ARGS
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (kPair) mbar_arrive_cluster(acce_leader0 + acc * 8);
        else mbar_arrive(acce + acc);
      }
    }
  }
  if (warp >= 2 && lane == 0) bulk_wait0();  // stores complete before the CTA retires
  tc_fence_before();
  __syncwarp();
  // the leader's MMAs into the peer's TMEM, and the peer's remote arrivals on
  // the leader's barriers, are done before either CTA frees TMEM or exits
  if (kPair) cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (kPair) tmem_dealloc_pair(tmem_base, C::kTmemCols);
    else tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// Persistent grid: at most one CTA (or CTA pair) per SM that can hold one
// (launch_gemm then trims it to the fewest units that take as many rounds of
// tiles). Pairs need two SMs of one GPC, so their count comes from the
// occupancy calculator (cached per kernel and device).
template <typename Kern>
int persistent_units(Kern kern, bool pair, size_t smem, int threads, int* units) {
  static int cache[2][64] = {};
  int dev = 0;
  LLMK_CUDA(cudaGetDevice(&dev));
  if (dev >= 64) dev = 63;
  int& c = cache[pair ? 1 : 0][dev];
  if (c == 0) {
    if (!pair) {
      c = num_sms();
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * num_sms());
      cfg.blockDim = dim3(threads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = num_sms() / 2;
      }
      c = std::min(clusters, num_sms() / 2);
    }
  }
  *units = c;
  return LLMK_OK;
}

template <bool kTF32, bool kAMN, bool kBMN, int kBN, bool kPair, int kOp>
int launch_gemm(const void* A, long long lda, const void* B, long long ldb, int M, int N, int K, EpiParams ep,
                int splits, cudaStream_t stream) {
  using C = Cfg<kTF32, kAMN, kBMN, kBN, kPair, op_bufs(kOp)>;
  auto kern = gemm_tc_kernel<kTF32, kAMN, kBMN, kBN, kPair, kOp>;
  static bool attr_done[64] = {};
  int dev = 0;
  LLMK_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !attr_done[dev]) {
    LLMK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM)));
    attr_done[dev] = true;
  }
  const CUtensorMapDataType dt = kTF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta, tb;
  const CUtensorMapSwizzle mn_swz = kTF32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  if (!kAMN) LLMK_TRY(make_tmap_2d(&ta, A, dt, K, M, lda * C::kElem, C::BK, C::BM));
  else LLMK_TRY(make_tmap_2d(&ta, A, dt, M, K, lda * C::kElem, C::kAtomMN, C::BK, mn_swz));
  if (!kBMN) LLMK_TRY(make_tmap_2d(&tb, B, dt, K, N, ldb * C::kElem, C::BK, C::BNC));
  else LLMK_TRY(make_tmap_2d(&tb, B, dt, N, K, ldb * C::kElem, C::kAtomMN, C::BK, mn_swz));
  CUtensorMap td;
  if (ep.partial) {
    LLMK_TRY(make_tmap_3d(&td, ep.partial, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M, splits, static_cast<uint64_t>(N) * 4,
                          static_cast<uint64_t>(M) * N * 4, 32, 32, 1));
  } else if (ep.d_bf16) {
    LLMK_TRY(make_tmap_2d(&td, ep.D, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, N, M, ep.ldd * 2, 64, 32));
  } else {
    LLMK_TRY(make_tmap_2d(&td, ep.D, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M, ep.ldd * 4, 32, 32));
  }
  // GELU pre-activation map (same chunk boxes as D); for the operand-loading
  // programs the residual's or the pre-activation's load map, with D's chunk
  // box; a copy of D's otherwise
  CUtensorMap tx = td;
  if constexpr (kOp == kOpBiasRes) {
    LLMK_TRY(make_tmap_2d(&tx, ep.residual, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M, ep.ldr * 4, 32, 32));
  } else if constexpr (kOp == kOpGeluBwd) {
    if (ep.d_bf16) LLMK_TRY(make_tmap_2d(&tx, ep.aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, N, M, ep.ldaux * 2, 64, 32));
    else LLMK_TRY(make_tmap_2d(&tx, ep.aux, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M, ep.ldaux * 4, 32, 32));
  } else if (ep.aux_tma) {
    if (ep.d_bf16) LLMK_TRY(make_tmap_2d(&tx, ep.aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, N, M, ep.ldaux * 2, 64, 32));
    else LLMK_TRY(make_tmap_2d(&tx, ep.aux, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, N, M, ep.ldaux * 4, 32, 32));
  }
  const int num_m = (M + C::kMmaM - 1) / C::kMmaM;
  const int num_tiles = num_m * ((N + kBN - 1) / kBN) * splits;
  // raster group (tile rows): one group over all of M when B is large (> 32 MB,
  // so it would be re-read from DRAM once per group) and A fits in L2 (<= 32 MB)
  const double a_bytes = static_cast<double>(M) * K * C::kElem, b_bytes = static_cast<double>(N) * K * C::kElem;
  const int group_m = (b_bytes > 32e6 && a_bytes <= 32e6) ? num_m : std::min(8, num_m);
  int units = 0;
  LLMK_TRY(persistent_units(kern, kPair, C::SMEM, C::kThreads, &units));
  // the fewest CTAs (pairs) that take as many rounds of tiles as all of them
  // would, when that frees at most 15 % of them: the rest of the SMs stay free
  // for work on other streams and leave power for a higher clock. Trimming
  // more (GPT-2 774M's 160- and 75-tile shapes: 54 and 38 of 74 pairs) made
  // its training step slower.
  const int rounds = (num_tiles + units - 1) / units;
  const int trimmed = (num_tiles + rounds - 1) / rounds;
  if (20 * trimmed >= 17 * units) units = trimmed;
  else units = std::min(units, num_tiles);
  unsigned int* st = device_status_ptr();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kPair) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * units);
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LLMK_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, td, tx, ep, M, N, K, splits, group_m, st));
  } else {
    kern<<<units, C::kThreads, C::SMEM, s>>>(ta, tb, td, tx, ep, M, N, K, splits, group_m, st);
  }
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

// Picks the kernel for the operand majorness and the epilogue program. The
// specialised programs are instantiated for the CTA-pair kernels where the
// training step uses them (forward: bias, bias + residual, bias + GELU;
// input gradient: GELU-backward; every form: plain store and split-K
// partials); everything else runs the flag-driven program.
template <bool kTF32, int kBN, bool kPair>
int dispatch_major(int a_trans, int b_trans, const void* A, long long lda, const void* B, long long ldb, int M,
                   int N, int K, const EpiParams& ep, int splits, cudaStream_t s) {
  // row statistics: only the logits GEMM (both operands K-major) takes them
  if (ep.stats) {
    if (a_trans || b_trans) return fail(LLMK_ERR_UNSUPPORTED, "gemm: row statistics need K-major operands");
    return launch_gemm<kTF32, false, false, kBN, kPair, kOpStats>(A, lda, B, ldb, M, N, K, ep, splits, s);
  }
  if (!a_trans && !b_trans) {
    if constexpr (kPair) {
      switch (ep.op) {
        case kOpNone: return launch_gemm<kTF32, false, false, kBN, kPair, kOpNone>(A, lda, B, ldb, M, N, K, ep, splits, s);
        case kOpBias: return launch_gemm<kTF32, false, false, kBN, kPair, kOpBias>(A, lda, B, ldb, M, N, K, ep, splits, s);
        case kOpBiasRes:
          return launch_gemm<kTF32, false, false, kBN, kPair, kOpBiasRes>(A, lda, B, ldb, M, N, K, ep, splits, s);
        case kOpBiasGelu:
          return launch_gemm<kTF32, false, false, kBN, kPair, kOpBiasGelu>(A, lda, B, ldb, M, N, K, ep, splits, s);
        default: break;
      }
    }
    return launch_gemm<kTF32, false, false, kBN, kPair, kOpGeneric>(A, lda, B, ldb, M, N, K, ep, splits, s);
  }
  if (!a_trans && b_trans) {
    if constexpr (kPair) {
      if (ep.op == kOpNone) return launch_gemm<kTF32, false, true, kBN, kPair, kOpNone>(A, lda, B, ldb, M, N, K, ep, splits, s);
      if (ep.op == kOpGeluBwd)
        return launch_gemm<kTF32, false, true, kBN, kPair, kOpGeluBwd>(A, lda, B, ldb, M, N, K, ep, splits, s);
    }
    return launch_gemm<kTF32, false, true, kBN, kPair, kOpGeneric>(A, lda, B, ldb, M, N, K, ep, splits, s);
  }
  if (a_trans && b_trans) {
    if constexpr (kPair) {
      if (ep.op == kOpNone) return launch_gemm<kTF32, true, true, kBN, kPair, kOpNone>(A, lda, B, ldb, M, N, K, ep, splits, s);
    }
    return launch_gemm<kTF32, true, true, kBN, kPair, kOpGeneric>(A, lda, B, ldb, M, N, K, ep, splits, s);
  }
  return launch_gemm<kTF32, true, false, kBN, kPair, kOpGeneric>(A, lda, B, ldb, M, N, K, ep, splits, s);
}

}  // namespace
}  // namespace llmk
