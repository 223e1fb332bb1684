// Causal flash attention (head size 64, bf16 in / fp32 accumulate) on tcgen05.
//
// Reference: gpt2cuda::BatchCausalAttentionForward / Backward
// (gpt2/cuda/attention.cu:119-148) -> FA-2 CuTe kernels on mma.sync with one
// CTA per (batch, head) walking every query tile (kernel/flash_attn/
// flash_fwd_kernel.cuh:11-400, flash_bwd_kernel.cuh:94-480).
//
// Layout: qkv is the packed (B, T, 3C) activation; head h of Q/K/V is the
// 64-column slice at h*64 of the first/second/third C block. One 3D TMA map
// {3C, T, B} with a {64, 128, 1} box serves Q, K, V, dO and O tiles: rows past
// T of a batch read as zeros.
//
// Forward: persistent, one CTA per SM walking (pair of 128-query tiles,
// head, batch) items heaviest first; warp 0 = TMA, warp 1 = tcgen05 issuer
// (S = Q K^T into TMEM, O += P V in TMEM), warps 2..9 = softmax of the two
// tiles (thread = query row): exp2 online softmax with lazy rescaling, P ->
// TMEM (16-bit pairs, the P V MMA's A operand). The two tiles share each K/V load and
// take turns on the tensor core, so one's softmax overlaps the other's MMAs.
//
// Backward: persistent, one CTA per SM walking (128-key tile, head, batch)
// items; each walks query tiles from the diagonal down. S = Q K^T and
// dP = dO V^T land in TMEM (lane = query); 8 softmax warps (2 per TMEM lane
// quarter, 64 key columns each; thread = query row, so LSE and D are one value
// a thread) form P and dS = P (dP - D) in registers and then in smem once the
// previous tile's gradient MMAs are done; dV += P^T dO and dK += dS^T Q (P, dS
// read as M-major A operands) accumulate in TMEM, dQ_i = dS K lands in one of two TMEM
// buffers and is staged in smem and added to an fp32 workspace by TMA
// reduce-adds (issued by a warp of their own) while the next query tile runs. D = rowsum(dO * O) and the
// final dQ scaling run as small pre/post kernels.
#include <algorithm>
#include <type_traits>
#include <vector>

#include "ptx.cuh"
#include "runtime.h"

namespace llmk {
namespace {

constexpr int HD = 64;          // head size
constexpr int TILE = 128;       // query / key tile
constexpr int TILE_BYTES = TILE * HD * 2;  // 16 KB: one [128 x 64] bf16 tile, 128B rows

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 1024B-aligned
// 128B-swizzled atom column (TMA SWIZZLE_128B / UMMA SWIZZLE_128B pattern).
__device__ __forceinline__ uint32_t sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// ------------------------------------------------------------------ forward
// Work item w of the attention kernels: query-tile pair (forward) or key
// tile (backward) `tile` of head bh. Items are ordered by decreasing work.
struct AttnItem {
  int tile, b, h, bh;
};
__device__ __forceinline__ AttnItem fwd_item(int w, int nq, int B, int NH) {
  const int bh_count = B * NH;
  AttnItem it;
  it.tile = nq - 1 - w / bh_count;  // most key tiles first
  it.bh = w % bh_count;
  it.b = it.bh / NH;
  it.h = it.bh % NH;
  return it;
}

// The k-th item of this CTA in the persistent kernels' static schedule:
// rounds of gridDim.x items, alternate rounds in reverse CTA order (items are
// sorted by decreasing work, so a CTA that takes a heavy item in one round
// takes a light one in the next). n_items when the CTA has no k-th item.
__device__ __forceinline__ int sched_slot(int k, int n_items) {
  const int g = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
  const int w = k * g + ((k & 1) ? g - 1 - c : c);
  return w < n_items ? w : n_items;
}

// The last round of a schedule whose items do not fill it: CTA c takes the
// item of rank slot[c] in that round (-1: none), so the round's items go to
// the CTAs with the least work after the full rounds. Filled on the host.
constexpr int kMaxTailCtas = 256;
struct SchedTail {
  int16_t slot[kMaxTailCtas];
};

__device__ __forceinline__ int sched_slot_tail(int k, int n_items, int tail) {
  const int g = static_cast<int>(gridDim.x), full = n_items / g;
  if (k < full) return sched_slot(k, n_items);
  return (k == full && tail >= 0) ? full * g + tail : n_items;
}

// ------------------------------------------------------------------ forward
// CTA = 10 warps: warp 0 TMA, warp 1 tcgen05 issuer, warps 2..5 the softmax
// of query tile A = 2p of pair item p, warps 6..9 of tile B = 2p+1 (thread =
// query row = TMEM lane). Both tiles of a pair belong to one (batch, head)
// and share every K/V tile the TMA brings in (B needs one more: its
// diagonal). Each tile has one S buffer (128 TMEM columns) and one O
// accumulator (64 columns) in TMEM and its P tile in TMEM too (64 columns of
// 16-bit pairs, the A operand of the P V MMA read straight from tensor memory);
// the issuer serves the two tiles (S_x(j+1) once S_x(j) is read, PV_x(j) once
// P_x(j) is written) in the order their barriers complete, so one tile's
// softmax runs while the other's MMAs do.
struct FwdSmem {
  static constexpr int kStages = 3;
  static constexpr int Q_OFF = 0;                                  // 2 items x (Q_A, Q_B)
  static constexpr int KV_OFF = 4 * TILE_BYTES;                    // stages x (K, V)
  static constexpr int BAR_OFF = KV_OFF + kStages * 2 * TILE_BYTES;  // (P_A, P_B live in TMEM)
  static constexpr size_t BYTES = BAR_OFF + 256 + 1024;
};
constexpr int kFwdThreads = 320;
// TMEM columns of the forward: tile x has S at 192x (128 columns) and O at
// 192x + 128 (64 columns); P_x (bf16/fp16 pairs, the A operand of P V) at
// kFwdPCol + 64x.
constexpr uint32_t kFwdPCol = 384;

template <bool kF16>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, void* __restrict__ out_ptr, int out_f32,
                    float* __restrict__ lse, int B, int T, int NH, int C, unsigned int* status,
                    const __grid_constant__ SchedTail tail) {
  using S = FwdSmem;
  const int tail_slot = tail.slot[blockIdx.x];
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + S::Q_OFF;
  uint8_t* sKV = smem + S::KV_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* q_full = bars;                       // [item parity][A, B]
  uint64_t* q_empty = q_full + 4;                // [item parity][A, B]
  uint64_t* kv_full = q_empty + 4;               // [stages]
  uint64_t* kv_empty = kv_full + S::kStages;     // [stages]
  uint64_t* s_full = kv_empty + S::kStages;      // [A, B]
  uint64_t* p_full = s_full + 2;                 // [A, B]
  uint64_t* pv_done = p_full + 2;                // [A, B]: the tile's latest P V is done
  uint64_t* s_free = pv_done + 2;                // [A, B]: the softmax has read S
  uint64_t* done = s_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int nq = (T + TILE - 1) / TILE;
  const int np = (nq + 1) / 2;
  const int n_items = np * B * NH;
  // this CTA's k-th item (n_items: none)
  auto slot = [&](int k) { return sched_slot_tail(k, n_items, tail_slot); };
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(q_full + i, 1);
      mbar_init(q_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(p_full + i, 128);
      mbar_init(pv_done + i, 1);
      mbar_init(s_free + i, 128);
    }
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns of tile X (0 = A, 1 = B): S at 192X .. 192X+127, O at
  // 192X+128 .. 192X+191. Barrier phases follow counters every role keeps
  // alike: items n (Q buffers n&1), K/V tiles over all items (stages), and
  // per tile the key tiles processed so far (s_full / p_full / pv_done).

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_qkv);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int n = 0;
      for (int w = slot(0); w < n_items && ok; w = slot(n + 1), ++n) {
        const AttnItem it = fwd_item(w, np, B, NH);
        const int p = it.tile;
        const bool has_b = 2 * p + 1 < nq;
        const int nkv = 2 * p + 1 + (has_b ? 1 : 0);
        for (int x = 0; x < 2; ++x) {
          // tile B of an odd last pair lies past T and reads as zeros
          const int qb = (n & 1) * 2 + x;
          if (!mbar_wait(q_empty + qb, ((n >> 1) & 1) ^ 1u, status, abort_flag, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(q_full + qb, TILE_BYTES);
          tma_load_3d(sQ + qb * TILE_BYTES, &tm_qkv, q_full + qb, it.h * HD, (2 * p + x) * TILE, it.b);
        }
        for (int j = 0; j < nkv && ok; ++j) {
          if (!mbar_wait(kv_empty + stage, phase ^ 1u, status, abort_flag, 1)) { ok = false; break; }
          uint8_t* sK = sKV + stage * 2 * TILE_BYTES;
          mbar_arrive_expect_tx(kv_full + stage, 2 * TILE_BYTES);
          tma_load_3d(sK, &tm_qkv, kv_full + stage, C + it.h * HD, j * TILE, it.b);
          tma_load_3d(sK + TILE_BYTES, &tm_qkv, kv_full + stage, 2 * C + it.h * HD, j * TILE, it.b);
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S = Q K^T: M=128 queries, N=128 keys, both K-major (hd contiguous).
      constexpr uint32_t kFmt = kF16 ? kFmtF16 : kFmtBF16;
      const uint32_t idesc_s = idesc_f32acc(128, 128, kFmt, false, false);
      // O += P V: M=128 queries, N=64 hd, K=128 keys; V is [keys][hd] = N-major.
      const uint32_t idesc_o = idesc_f32acc(128, HD, kFmt, false, true);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t cp[2] = {0, 0};  // P tiles consumed per query tile
      uint32_t cf[2] = {0, 0};  // S tiles released per query tile
      bool ok = true;
      int n = 0;
      auto issue_s = [&](int x, int st, int qb) {
        const uint32_t q_addr = smem_u32(sQ + qb * TILE_BYTES);
        const uint32_t k_addr = smem_u32(sKV + st * 2 * TILE_BYTES);
        const uint32_t d = tmem + x * 192;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_f16_ss(d, sdesc_sw128(q_addr + ks * 32, 16, 1024), sdesc_sw128(k_addr + ks * 32, 16, 1024), idesc_s,
                     ks > 0);
        mma_commit(s_full + x);
      };
      auto issue_pv = [&](int x, int st, bool acc) {
        // A = P_x in TMEM (columns 384 + 64x: 128 keys as 64 packed pairs), 16 keys a K-step
        const uint32_t p_tmem = tmem + kFwdPCol + x * (TILE / 2);
        const uint32_t v_addr = smem_u32(sKV + st * 2 * TILE_BYTES + TILE_BYTES);
        const uint32_t d = tmem + x * 192 + 128;
#pragma unroll
        for (int ks = 0; ks < TILE / 16; ++ks) {
          const uint64_t bd = sdesc_sw128(v_addr + ks * 2048, TILE_BYTES, 1024);
          mma_f16_ts(d, p_tmem + ks * 8, bd, idesc_o, (ks > 0 || acc) ? 1u : 0u);
        }
        mma_commit(pv_done + x);
      };
      for (int w = slot(0); w < n_items && ok; w = slot(n + 1), ++n) {
        const AttnItem it = fwd_item(w, np, B, NH);
        const int p = it.tile;
        const bool has_b = 2 * p + 1 < nq;
        const int na = 2 * p + 1, nkv = na + (has_b ? 1 : 0);
        const int q0 = (n & 1) * 2;
        if (!mbar_wait(q_full + q0, (n >> 1) & 1, status, abort_flag, 2) ||
            !mbar_wait(q_full + q0 + 1, (n >> 1) & 1, status, abort_flag, 2)) { ok = false; break; }
        if (!mbar_wait(kv_full + stage, phase, status, abort_flag, 3)) { ok = false; break; }
        tc_fence_after();
        // S_x(k) is issued as soon as the softmax has read S_x(k-1), ahead of
        // P V_x(k-1); after the tile's last S its Q buffer is free.
        issue_s(0, stage, q0);
        if (na == 1) mma_commit(q_empty + q0);
        if (has_b) issue_s(1, stage, q0 + 1);
        for (int j = 0; j < nkv; ++j) {
          const int st = stage;
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
          bool next_ready = false;  // K/V tile j+1 (now at `stage`) has landed
          // S_x(j+1) once the softmax has read S_x(j), P V_x(j) once P_x(j) is
          // in TMEM: each issued as soon as its barrier completes, whichever
          // tile comes first
          bool need_s[2], need_pv[2];
          int nxs[2];
          for (int x = 0; x < 2; ++x) {
            nxs[x] = x == 0 ? na : (has_b ? nkv : 0);
            need_s[x] = need_pv[x] = j < nxs[x];
          }
          const long long c0 = clock64();
          unsigned int polls = 0;
          while (ok && (need_s[0] || need_s[1] || need_pv[0] || need_pv[1])) {
            bool progressed = false;
            for (int x = 0; x < 2; ++x) {
              if (need_s[x] && mbar_peek(s_free + x, cf[x] & 1u)) {
                ++cf[x];
                need_s[x] = false;
                progressed = true;
                if (j + 1 < nxs[x]) {
                  if (!next_ready) {
                    if (!mbar_wait(kv_full + stage, phase, status, abort_flag, 3)) { ok = false; break; }
                    next_ready = true;
                  }
                  tc_fence_after();
                  issue_s(x, stage, q0 + x);
                  if (j + 2 == nxs[x]) mma_commit(q_empty + q0 + x);
                }
              }
              if (need_pv[x] && !need_s[x] && mbar_peek(p_full + x, cp[x] & 1u)) {
                ++cp[x];
                need_pv[x] = false;
                progressed = true;
                tc_fence_after();
                issue_pv(x, st, j > 0);
              }
            }
            if (!ok || progressed) continue;
            if (*abort_flag || clock64() - c0 > kWaitLimitCycles || ++polls > kWaitLimitIters) {
              if (!*abort_flag) atomicOr(status, LLMK_DEV_TIMEOUT | (1u << (8 + 4)));
              *abort_flag = 1;
              ok = false;
            }
          }
          if (!ok) break;
          mma_commit(kv_empty + st);  // K_j, V_j read by every MMA issued so far
        }
        // tile B of an odd last pair: its (zero) Q buffer is free
        if (ok && !has_b) mma_commit(q_empty + q0 + 1);
      }
      mma_commit(done);
      mbar_wait(done, 0, status, nullptr, 5);
    }
    __syncwarp();
  } else {
    const int x = (warp - 2) >> 2;  // query tile of the pair
    const int q = warp & 3;
    const int r = q * 32 + lane;  // query row within the tile (= TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t s_cols = tmem + lane_base + x * 192;
    const uint32_t o_cols = s_cols + 128;
    const uint32_t p_cols = tmem + lane_base + kFwdPCol + x * (TILE / 2);
    const float sl2 = 0.125f * 1.4426950408889634f;  // softmax scale * log2(e)
    // O accumulates P V over the tile's key tiles in TMEM. Exponents use a
    // running reference m (log2 domain) that moves only when a tile's row
    // maximum exceeds it by more than kRescale: then the warp rescales its O
    // rows and l in place once the previous P V is done. Otherwise P stays
    // below 2^kRescale, well inside bf16 and fp32 range.
    constexpr float kRescale = 8.f;
    bool ok = true;
    uint32_t cs = 0;  // S tiles consumed
    int n = 0;        // items
    for (int w = slot(0); w < n_items && ok; w = slot(n + 1), ++n) {
      const AttnItem it = fwd_item(w, np, B, NH);
      const int tile = 2 * it.tile + x;
      if (tile >= nq) continue;  // tile B of an odd last pair
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j <= tile; ++j) {
        bool wt = mbar_wait(s_full + x, cs & 1u, status, abort_flag, 6);
        ++cs;
        if (!__all_sync(0xffffffffu, wt)) { ok = false; break; }
        tc_fence_after();
        // the row's 128 scores in registers; S_x is then free for the next tile
        uint32_t sv[TILE];
#pragma unroll
        for (int c = 0; c < TILE; c += 32)
          tmem_ld_32x32b_x32(s_cols + c, *reinterpret_cast<uint32_t(*)[32]>(sv + c));
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(s_free + x);
        if (j == tile) {  // diagonal tile: key index > query index is masked
#pragma unroll
          for (int i = 0; i < TILE; ++i)
            if (i > r) sv[i] = __float_as_uint(-INFINITY);
        }
        // row max (raw scores; the scale is positive) as a tree
        float mx4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) mx4[k] = __uint_as_float(sv[k]);
#pragma unroll
        for (int i = 4; i < TILE; i += 4)
#pragma unroll
          for (int k = 0; k < 4; ++k) mx4[k] = fmaxf(mx4[k], __uint_as_float(sv[i + k]));
        const float mx2 = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
        // P V of the previous S tile (of this or the previous item) must be
        // done before O is rescaled or P overwritten
        if (cs > 1) {
          bool wp = mbar_wait(pv_done + x, (cs - 2) & 1u, status, abort_flag, 7);
          if (!__all_sync(0xffffffffu, wp)) { ok = false; break; }
          tc_fence_after();
        }
        const bool move = mx2 > m + kRescale;
        if (j > 0 && __any_sync(0xffffffffu, move)) {
          const float alpha = move ? ex2_approx(m - mx2) : 1.f;
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            uint32_t ov[16];
            tmem_ld_32x32b_x16(o_cols + c, ov);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st_32x32b_x16(o_cols + c, ov);
          }
          tmem_st_wait();
          l *= alpha;
        }
        if (move) m = mx2;
        // P = 2^(S * scale * log2e - m) two columns at a time (packed fp32
        // pairs), row sum in 8 running partial sums (4 packed pairs)
        const uint64_t sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m, -m);
        uint64_t rs2[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) rs2[k] = f2_pack(0.f, 0.f);
#pragma unroll
        for (int ch = 0; ch < TILE / 8; ++ch) {
          uint32_t pk[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int i = ch * 8 + 2 * k;
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1])), sl2x2, negm2), x0, x1);
            const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            rs2[k] = f2_add(rs2[k], f2_pack(p0, p1));
            pk[k] = pack16x2<kF16>(p0, p1);
          }
          tmem_st_32x32b_x4(p_cols + ch * 4, pk[0], pk[1], pk[2], pk[3]);
        }
        float rs8[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) f2_unpack(rs2[k], rs8[2 * k], rs8[2 * k + 1]);
        l += ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full + x);
      }
      if (!ok) break;
      // the tile's last P V, then O / l
      bool wo = mbar_wait(pv_done + x, (cs - 1) & 1u, status, abort_flag, 7);
      if (!__all_sync(0xffffffffu, wo)) { ok = false; break; }
      tc_fence_after();
      uint32_t ov[HD];
      tmem_ld_32x32b_x32(o_cols, *reinterpret_cast<uint32_t(*)[32]>(ov));
      tmem_ld_32x32b_x32(o_cols + 32, *reinterpret_cast<uint32_t(*)[32]>(ov + 32));
      tmem_ld_wait();
      const int t = tile * TILE + r;
      if (t < T) {
        const float inv = 1.0f / l;
        const long long off = (static_cast<long long>(it.b) * T + t) * C + it.h * HD;
        if (out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out_ptr) + off);
#pragma unroll
          for (int ch = 0; ch < HD / 4; ++ch)
            dst[ch] = make_float4(__uint_as_float(ov[ch * 4]) * inv, __uint_as_float(ov[ch * 4 + 1]) * inv,
                                  __uint_as_float(ov[ch * 4 + 2]) * inv, __uint_as_float(ov[ch * 4 + 3]) * inv);
        } else {
          uint16_t* dst = static_cast<uint16_t*>(out_ptr) + off;
#pragma unroll
          for (int ch = 0; ch < HD / 8; ++ch) {
            uint4 u;
            u.x = pack16x2<kF16>(__uint_as_float(ov[ch * 8 + 0]) * inv, __uint_as_float(ov[ch * 8 + 1]) * inv);
            u.y = pack16x2<kF16>(__uint_as_float(ov[ch * 8 + 2]) * inv, __uint_as_float(ov[ch * 8 + 3]) * inv);
            u.z = pack16x2<kF16>(__uint_as_float(ov[ch * 8 + 4]) * inv, __uint_as_float(ov[ch * 8 + 5]) * inv);
            u.w = pack16x2<kF16>(__uint_as_float(ov[ch * 8 + 6]) * inv, __uint_as_float(ov[ch * 8 + 7]) * inv);
            reinterpret_cast<uint4*>(dst)[ch] = u;
          }
        }
        // natural-log LSE: (m2 + log2 l) * ln 2
        lse[static_cast<long long>(it.bh) * T + t] = (m + __log2f(l)) * 0.6931471805599453f;
      }
      tc_fence_before();
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------- backward
__device__ __forceinline__ void load8f(const __nv_bfloat16* p, float* v) {
  uint4 a = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 u = __bfloat1622float2(x[i]);
    v[2 * i] = u.x;
    v[2 * i + 1] = u.y;
  }
}
__device__ __forceinline__ void load8f(const __half* p, float* v) {
  uint4 a = *reinterpret_cast<const uint4*>(p);
  const __half2* x = reinterpret_cast<const __half2*>(&a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 u = __half22float2(x[i]);
    v[2 * i] = u.x;
    v[2 * i + 1] = u.y;
  }
}
__device__ __forceinline__ void load8f(const float* p, float* v) {
  float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// D[b,h,t] = sum_i dO[b,t,h*64+i] * O[b,t,h*64+i] for every head of row
// (b,t), and zeroes the row's dq_acc. One warp per row: lane l reads the
// 16-byte chunks l, l+32, ... of dO and O (8 chunks per head, so each head's
// sum is a reduction over 8 consecutive lanes). With fp32 dO / O (IoT =
// float) it also writes the 16-bit copy of dO the MMAs read (dout16, fp16
// when kF16, else bf16).
template <typename IoT, bool kF16>
__global__ void __launch_bounds__(256) attn_bwd_pre_kernel(float* __restrict__ D, float* __restrict__ dq_acc,
                                                           uint16_t* __restrict__ dout16,
                                                           const IoT* __restrict__ dout, const IoT* __restrict__ o,
                                                           int B, int T, int NH, int C) {
  const long long bt = blockIdx.x * 8LL + (threadIdx.x >> 5);  // row (b, t)
  const int lane = threadIdx.x & 31;
  if (bt >= static_cast<long long>(B) * T) return;
  const int b = static_cast<int>(bt / T), t = static_cast<int>(bt % T);
  const IoT* pd = dout + bt * C;
  const IoT* po = o + bt * C;
  const int nchunk = C / 8;  // 8 per head
  for (int c0 = 0; c0 < nchunk; c0 += 32) {
    const int c = c0 + lane;
    float s = 0.f;
    if (c < nchunk) {
      float x[8], y[8];
      load8f(pd + 8 * c, x);
      load8f(po + 8 * c, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += x[i] * y[i];
      if constexpr (sizeof(IoT) == 4) {
        uint4 u;
        u.x = pack16x2<kF16>(x[0], x[1]);
        u.y = pack16x2<kF16>(x[2], x[3]);
        u.z = pack16x2<kF16>(x[4], x[5]);
        u.w = pack16x2<kF16>(x[6], x[7]);
        *reinterpret_cast<uint4*>(dout16 + bt * C + 8 * c) = u;
      }
    }
    // the 8 lanes of a head: fixed-order butterfly
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if (c < nchunk && (c & 7) == 0) D[(static_cast<long long>(b) * NH + c / 8) * T + t] = s;
  }
  float4* z = reinterpret_cast<float4*>(dq_acc + bt * C);
  for (int k = lane; k < C / 4; k += 32) z[k] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// dqkv[:, :, 0:C] = dq_acc * scale (fp32, or 16-bit: fp16 when kF16, else bf16)
template <typename IoT, bool kF16>
__global__ void attn_bwd_post_kernel(IoT* __restrict__ dqkv, const float* __restrict__ dq_acc, int BT, int C,
                                     float scale) {
  const long long n8 = static_cast<long long>(BT) * C / 8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = i * 8;
    const long long bt = e / C;
    const int c = static_cast<int>(e - bt * C);
    const float4* p = reinterpret_cast<const float4*>(dq_acc + e);
    float4 a = p[0], bb = p[1];
    if constexpr (sizeof(IoT) == 4) {
      float4* d = reinterpret_cast<float4*>(dqkv + bt * 3 * C + c);
      d[0] = make_float4(a.x * scale, a.y * scale, a.z * scale, a.w * scale);
      d[1] = make_float4(bb.x * scale, bb.y * scale, bb.z * scale, bb.w * scale);
    } else {
      uint4 u;
      u.x = pack16x2<kF16>(a.x * scale, a.y * scale);
      u.y = pack16x2<kF16>(a.z * scale, a.w * scale);
      u.z = pack16x2<kF16>(bb.x * scale, bb.y * scale);
      u.w = pack16x2<kF16>(bb.z * scale, bb.w * scale);
      *reinterpret_cast<uint4*>(dqkv + bt * 3 * C + c) = u;
    }
  }
}

// The backward's buffers fill the 227 KB a CTA may use, leaving no room for a
// runtime alignment pad: the dynamic shared memory is declared 1024-byte
// aligned (the 128B-swizzle atom) and the kernel checks that it is.
struct BwdSmem {
  static constexpr int kStages = 2;
  // K, V of two items (by item parity: buffer b holds K at 2b tiles, V one
  // tile further), so the next item's K / V arrive while this item runs
  static constexpr int K_OFF = 0;
  static constexpr int KV_BYTES = 2 * TILE_BYTES;  // K, then V at + TILE_BYTES
  static constexpr int QD_OFF = 2 * KV_BYTES;                      // stages x (Q_i, dO_i)
  static constexpr int PD_OFF = QD_OFF + kStages * 2 * TILE_BYTES;  // P, dS [128 q x 128 keys]
  static constexpr int PD_BYTES = 4 * TILE_BYTES;
  static constexpr int DQ_OFF = PD_OFF + PD_BYTES;                 // dQ staging: 2 x [128 q x 32] fp32, 128B-swizzled
  static constexpr int LD_OFF = DQ_OFF + 2 * TILE_BYTES;           // stages x (LSE[128], D[128]) fp32
  static constexpr int BAR_OFF = LD_OFF + kStages * 2 * TILE * 4;
  static constexpr size_t BYTES = BAR_OFF + 256;
  static_assert(BYTES <= 232448, "backward smem");
};

// Backward CTA = 3 + kBwdSoftmaxWarps warps: warp 0 TMA, warp 1 tcgen05
// issuer, warps 2.. the softmax-gradient warps, the last warp the dQ
// reduce issuer. Softmax warp w reads TMEM lanes
// 32*(w%4).. (query rows of S / dP / dQ, key rows of dK / dV) and owns
// column group (w-2)/4 of every tile it touches: kBwdSoftmaxWarps/4 warps
// share each lane quarter and split its columns.
//
// A persistent CTA (one per SM) walks key-tile items in the snake-order
// schedule (sched_slot_tail; most query tiles first). The query-tile steps g of a
// CTA's items form one sequence. The softmax warps turn S / dP of step g into P /
// dS in registers while the gradient MMAs of step g-1 run, write them to
// the single smem P / dS buffer once those MMAs are done, and then stage
// dQ of step g-1 (TMEM, double-buffered by step parity) for the TMA
// reduce-adds into the fp32 accumulator, which the last warp issues once every
// softmax warp has staged its part: the softmax warps never wait for one
// another there, only (a step later) for those reduce-adds to have read the
// staging.
// Eight softmax warps (64 columns of each tile per warp, two per TMEM lane
// quarter): measured 3.6 % faster per call than sixteen at B = 16, T = 1024 —
// fewer arrivals per barrier phase and 168 registers a thread instead of the
// 96 that sixteen warps leave (which spill more).
#ifndef LLMK_BWD_SOFTMAX_WARPS
#define LLMK_BWD_SOFTMAX_WARPS 8
#endif
constexpr int kBwdSoftmaxWarps = LLMK_BWD_SOFTMAX_WARPS;  // 8 or 16
constexpr int kBwdDqWarp = 2 + kBwdSoftmaxWarps;            // the dQ reduce issuer
constexpr int kBwdThreads = 32 * (kBwdDqWarp + 1);
constexpr int kBwdCols = 4 * TILE / kBwdSoftmaxWarps;     // S key columns per warp (64 or 32)
constexpr int kBwdGradCols = HD * 4 / kBwdSoftmaxWarps;   // dQ / dK / dV columns per warp (32 or 16)
static_assert(kBwdSoftmaxWarps == 8 || kBwdSoftmaxWarps == 16, "softmax warps");

__device__ __forceinline__ AttnItem bwd_item(int w, int B, int NH) {
  const int bh_count = B * NH;
  AttnItem it;
  it.tile = w / bh_count;  // key tile kt: query tiles kt..nk-1, so kt = 0 first
  it.bh = w % bh_count;
  it.b = it.bh / NH;
  it.h = it.bh % NH;
  return it;
}

// P = exp2(S * scale*log2e - LSE*log2e) and dS = P (dP - D) for one
// thread's query row tq and kCols key columns tk0.., packed as pairs of the
// 16-bit operand type into pk / dk. nl2 = -LSE * log2e and d = D of the row.
// kMask: the diagonal tile (key > query masked) or a tile reaching past T
// (padded queries masked).
template <bool kMask, int kCols, bool kF16>
__device__ __forceinline__ void bwd_p_ds(const uint32_t* sv, const uint32_t* dv, float nl2, float d, int tk0, int tq,
                                         int T, uint32_t* pk, uint32_t* dk) {
  const float sl2 = 0.125f * kLog2e;
  const uint64_t sl2x2 = f2_pack(sl2, sl2), nl2x2 = f2_pack(nl2, nl2), dd = f2_pack(d, d);
#pragma unroll
  for (int h = 0; h < kCols / 2; ++h) {
    const int i = 2 * h;
    // x = S * scale * log2e - LSE * log2e, two columns at a time
    const uint64_t x = f2_fma(f2_pack(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1])), sl2x2, nl2x2);
    float x0, x1;
    f2_unpack(x, x0, x1);
    float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
    if (kMask) {  // causal (key after query) and padded queries
      const int tk = tk0 + i;
      if (tk > tq || tq >= T) p0 = 0.f;
      if (tk + 1 > tq || tq >= T) p1 = 0.f;
    }
    // dS = P (dP - D)
    const uint64_t pp = f2_pack(p0, p1);
    const uint64_t t = f2_fma(dd, f2_pack(-1.f, -1.f), f2_pack(__uint_as_float(dv[i]), __uint_as_float(dv[i + 1])));
    float d0, d1;
    f2_unpack(f2_mul(pp, t), d0, d1);
    pk[h] = pack16x2<kF16>(p0, p1);
    dk[h] = pack16x2<kF16>(d0, d1);
  }
}

template <bool kF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq,
                    void* __restrict__ dqkv_ptr, int io_f32, float* __restrict__ dq_acc,
                    const float* __restrict__ lse, const float* __restrict__ Dvec, int B, int T, int NH, int C,
                    unsigned int* status, const __grid_constant__ SchedTail tail) {
  using S = BwdSmem;
  const int tail_slot = tail.slot[blockIdx.x];
  extern __shared__ __align__(1024) uint8_t smem_bwd[];
  if ((smem_u32(smem_bwd) & 1023u) != 0) {  // uniform: every thread returns before any barrier
    if (threadIdx.x == 0) atomicOr(status, LLMK_DEV_SMEM_ALIGN);
    return;
  }
  uint8_t* smem = smem_bwd;
  uint8_t* sK = smem + S::K_OFF;
  uint8_t* sQD = smem + S::QD_OFF;
  uint8_t* sPD = smem + S::PD_OFF;  // P, dS 2 tiles further
  float* sLD = reinterpret_cast<float*>(smem + S::LD_OFF);
  uint8_t* sDQ = smem + S::DQ_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* kv_full = bars;                       // [2] K, V of an item of parity b loaded
  uint64_t* kv_empty = bars + 2;                  // [2] that item's last gradient MMAs done (buffer b free)
  uint64_t* qd_full = bars + 4;                   // [stages] Q_i, dO_i
  uint64_t* qd_empty = qd_full + S::kStages;      // [stages]
  uint64_t* sdp_full = qd_empty + S::kStages;     // S and dP in TMEM
  uint64_t* sdp_free = sdp_full + 1;              // S / dP read into registers (one arrival per warp)
  uint64_t* ps_full = sdp_free + 1;               // [2] P, dS of a step of parity b in smem
  uint64_t* grad_done = ps_full + 2;              // [2] gradient MMAs of step parity b done
  uint64_t* dq_free = grad_done + 2;              // [2] dQ TMEM buffer b read
  uint64_t* dkv_free = dq_free + 2;               // an item's dK / dV TMEM read
  uint64_t* ld_full = dkv_free + 1;               // [stages] LSE / D of a ring stage staged
  uint64_t* dqs_full = ld_full + S::kStages;      // dQ staging written (one arrival per softmax warp)
  uint64_t* dqs_free = dqs_full + 1;              // the previous dQ reduce-adds have read the staging
  uint64_t* done = dqs_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int nk = (T + TILE - 1) / TILE;
  const int n_items = nk * B * NH;
  // this CTA's k-th item (n_items: none)
  auto slot = [&](int k) { return sched_slot_tail(k, n_items, tail_slot); };
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(kv_full + b2, 1);
      mbar_init(kv_empty + b2, 1);
    }
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(qd_full + s, 1);
      mbar_init(qd_empty + s, 1);
      mbar_init(ld_full + s, 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(sdp_free, kBwdSoftmaxWarps);
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(ps_full + b2, kBwdSoftmaxWarps);
      mbar_init(grad_done + b2, 1);
      mbar_init(dq_free + b2, kBwdSoftmaxWarps);
    }
    mbar_init(dkv_free, kBwdSoftmaxWarps);
    mbar_init(dqs_full, kBwdSoftmaxWarps);
    mbar_init(dqs_free, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S 0..127, dP 128..255, dV 256..319, dK 320..383,
  // dQ[0] 384..447, dQ[1] 448..511

  if (warp == 0) {
    // lane 0 issues the TMA loads; all 32 lanes stage LSE (log2 units) and D
    // of each query tile next to its Q / dO ring stage (0 past T)
    if (lane == 0) {
      tma_prefetch_desc(&tm_qkv);
      tma_prefetch_desc(&tm_do);
    }
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int n = 0;
    for (int w = slot(0); w < n_items && ok; w = slot(n + 1), ++n) {
      const AttnItem it = bwd_item(w, B, NH);
      const int kt = it.tile, nqi = nk - kt;
      const float* lse_bh = lse + static_cast<long long>(it.bh) * T;
      const float* d_bh = Dvec + static_cast<long long>(it.bh) * T;
      {
        // K, V of this item into buffer n&1 once the item two back (its
        // previous user) has finished its gradient MMAs; this runs as soon as
        // the previous item's Q / dO loads are issued, a step or two ahead
        const int kb = n & 1;
        bool wt = mbar_wait(kv_empty + kb, ((n >> 1) & 1) ^ 1u, status, abort_flag, 19);
        if (!__all_sync(0xffffffffu, wt)) { ok = false; break; }
        if (lane == 0) {
          uint8_t* kv = sK + kb * S::KV_BYTES;
          mbar_arrive_expect_tx(kv_full + kb, 2 * TILE_BYTES);
          tma_load_3d(kv, &tm_qkv, kv_full + kb, C + it.h * HD, kt * TILE, it.b);
          tma_load_3d(kv + TILE_BYTES, &tm_qkv, kv_full + kb, 2 * C + it.h * HD, kt * TILE, it.b);
        }
      }
      for (int i = 0; i < nqi; ++i) {
        const int q0 = (kt + i) * TILE;
        bool wt = mbar_wait(qd_empty + stage, phase ^ 1u, status, abort_flag, 8);
        if (!__all_sync(0xffffffffu, wt)) { ok = false; break; }
        if (lane == 0) {
          uint8_t* sq = sQD + stage * 2 * TILE_BYTES;
          mbar_arrive_expect_tx(qd_full + stage, 2 * TILE_BYTES);
          tma_load_3d(sq, &tm_qkv, qd_full + stage, it.h * HD, q0, it.b);
          tma_load_3d(sq + TILE_BYTES, &tm_do, qd_full + stage, it.h * HD, q0, it.b);
        }
        // LSE and D of the tile's queries: two 512-byte bulk copies for a full,
        // 16-byte aligned tile (the common case), plain loads otherwise
        float* ld = sLD + stage * 2 * TILE;
        const bool bulk = q0 + TILE <= T && (reinterpret_cast<uintptr_t>(lse_bh + q0) & 15u) == 0 &&
                          (reinterpret_cast<uintptr_t>(d_bh + q0) & 15u) == 0;
        if (bulk) {
          if (lane == 0) {
            mbar_arrive_expect_tx(ld_full + stage, 2 * TILE * 4);
            bulk_load_1d(ld, lse_bh + q0, TILE * 4, ld_full + stage);
            bulk_load_1d(ld + TILE, d_bh + q0, TILE * 4, ld_full + stage);
          }
        } else {
          for (int k = lane; k < TILE; k += 32) {
            const int t = q0 + k;
            ld[k] = t < T ? lse_bh[t] : 0.f;
            ld[TILE + k] = t < T ? d_bh[t] : 0.f;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(ld_full + stage);
        }
        if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S = Q K^T and dP = dO V^T: M=128 q, N=128 keys, K=64 (all K-major).
      constexpr uint32_t kFmt = kF16 ? kFmtF16 : kFmtBF16;
      const uint32_t idesc_s = idesc_f32acc(128, 128, kFmt, false, false);
      // dV += P^T dO, dK += dS^T Q: M=128 keys, N=64, K=128 q; A = P / dS stored
      // [q][keys] = M-major; B is [q][hd] = N-major.
      const uint32_t idesc_kv = idesc_f32acc(128, HD, kFmt, true, true);
      // dQ = dS K: M=128 q, N=64, K=128 keys; A = dS stored [q][keys] = K-major;
      // B = K stored [keys][hd] = N-major.
      const uint32_t idesc_q = idesc_f32acc(128, HD, kFmt, false, true);
      auto issue_sdp = [&](int st, int kb) {
        const uint32_t k_addr = smem_u32(sK) + kb * S::KV_BYTES, v_addr = k_addr + TILE_BYTES;
        const uint32_t q_addr = smem_u32(sQD + st * 2 * TILE_BYTES);
        const uint32_t do_addr = q_addr + TILE_BYTES;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_f16_ss(tmem + 0, sdesc_sw128(q_addr + ks * 32, 16, 1024), sdesc_sw128(k_addr + ks * 32, 16, 1024),
                     idesc_s, ks > 0);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_f16_ss(tmem + 128, sdesc_sw128(do_addr + ks * 32, 16, 1024), sdesc_sw128(v_addr + ks * 32, 16, 1024),
                     idesc_s, ks > 0);
        mma_commit(sdp_full);
      };
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;
      bool issued = false;  // S / dP of step g already issued
      int n = 0;
      for (int w = slot(0); w < n_items && ok; w = slot(n + 1), ++n) {
        const int nqi = nk - bwd_item(w, B, NH).tile;
        const int kb = n & 1;
        const bool has_next = slot(n + 1) < n_items;
        const uint32_t k_addr = smem_u32(sK) + kb * S::KV_BYTES;
        for (int j = 0; j < nqi; ++j, ++g) {
          const int nst = stage + 1 == S::kStages ? 0 : stage + 1;
          const uint32_t nph = stage + 1 == S::kStages ? phase ^ 1u : phase;
          const uint32_t pb = g & 1;
          if (!issued) {
            // first step of an item: its K, V, and the S / dP TMEM of the previous step
            if ((j == 0 && !mbar_wait(kv_full + kb, (n >> 1) & 1, status, abort_flag, 9)) ||
                !mbar_wait(qd_full + stage, phase, status, abort_flag, 10) ||
                (g > 0 && !mbar_wait(sdp_free, (g - 1) & 1, status, abort_flag, 11))) { ok = false; break; }
            tc_fence_after();
            issue_sdp(stage, kb);
          }
          issued = false;
          if (j + 1 < nqi || has_next) {
            // the next step, of this item or the first of the next one (its K, V
            // in the other buffer), as soon as the softmax warps hold this one
            // in registers
            const int nkb = j + 1 < nqi ? kb : kb ^ 1;
            if (!mbar_wait(sdp_free, g & 1, status, abort_flag, 11) ||
                !mbar_wait(qd_full + nst, nph, status, abort_flag, 10) ||
                (j + 1 == nqi && !mbar_wait(kv_full + nkb, ((n + 1) >> 1) & 1, status, abort_flag, 9))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_sdp(nst, nkb);
            issued = true;
          }
          // P / dS of this step in smem; dQ buffer pb read (step g-2); at an
          // item's first step, the previous item's dK / dV read
          if (!mbar_wait(ps_full + pb, (g >> 1) & 1, status, abort_flag, 12) ||
              (g >= 2 && !mbar_wait(dq_free + pb, ((g >> 1) & 1) ^ 1u, status, abort_flag, 13)) ||
              (j == 0 && !mbar_wait(dkv_free, (n & 1) ^ 1u, status, abort_flag, 14))) { ok = false; break; }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQD + stage * 2 * TILE_BYTES);
          const uint32_t do_addr = q_addr + TILE_BYTES;
          const uint32_t p_addr = smem_u32(sPD), ds_addr = p_addr + 2 * TILE_BYTES;
          // dV, dK: A = P^T / dS^T as M-major from P / dS [q][keys] (key atoms 16 KB
          // apart, q groups 1 KB apart), K-step = 16 q rows.
#pragma unroll
          for (int ks = 0; ks < TILE / 16; ++ks) {
            mma_f16_ss(tmem + 256, sdesc_sw128(p_addr + ks * 2048, TILE_BYTES, 1024),
                       sdesc_sw128(do_addr + ks * 2048, TILE_BYTES, 1024), idesc_kv, (j > 0 || ks > 0));
            mma_f16_ss(tmem + 320, sdesc_sw128(ds_addr + ks * 2048, TILE_BYTES, 1024),
                       sdesc_sw128(q_addr + ks * 2048, TILE_BYTES, 1024), idesc_kv, (j > 0 || ks > 0));
          }
          // dQ = dS K: A = dS K-major (K = keys), K-step = 16 keys.
#pragma unroll
          for (int ks = 0; ks < TILE / 16; ++ks) {
            const uint32_t koff = (ks >> 2) * TILE_BYTES + (ks & 3) * 32;  // K (= key) offset in a [128 x 128] K-major tile
            mma_f16_ss(tmem + 384 + pb * HD, sdesc_sw128(ds_addr + koff, 16, 1024),
                       sdesc_sw128(k_addr + ks * 2048, TILE_BYTES, 1024), idesc_q, ks > 0);
          }
          mma_commit(grad_done + pb);
          mma_commit(qd_empty + stage);
          if (j + 1 == nqi) mma_commit(kv_empty + kb);
          stage = nst;
          phase = nph;
        }
      }
      mma_commit(done);
      mbar_wait(done, 0, status, nullptr, 5);
    }
    __syncwarp();
  } else if (warp == kBwdDqWarp) {
    // dQ of every step, in the softmax warps' step order: once all of them
    // have staged it (dqs_full), two TMA reduce-adds into the fp32
    // accumulator; once those have read the staging, dqs_free.
    if (lane == 0) {
      uint32_t f = 0;
      bool ok = true;
      int n = 0;
      for (int w = slot(0); w < n_items && ok; w = slot(++n)) {
        const AttnItem it = bwd_item(w, B, NH);
        for (int qt = it.tile; qt < nk; ++qt, ++f) {
          if (!mbar_wait(dqs_full, f & 1, status, abort_flag, 24)) { ok = false; break; }
          tma_reduce_add_3d(&tm_dq, sDQ, it.h * HD, qt * TILE, it.b);
          tma_reduce_add_3d(&tm_dq, sDQ + TILE_BYTES, it.h * HD + 32, qt * TILE, it.b);
          bulk_commit();
          bulk_wait_read0();
          mbar_arrive(dqs_free);
        }
      }
      bulk_wait0();  // the reduce-adds are complete before the CTA exits
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int cq = (warp - 2) >> 2;  // column quarter
    const int r = q * 32 + lane;     // query row within the tile for S/dP/dQ; key row for dK/dV
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // dQ of step gg (TMEM buffer gg&1, lane = query row, columns cq*16..+16)
    // staged in smem (two 128B-swizzled [128 x 32] fp32 halves) by all the
    // softmax warps, then added to the fp32 accumulator by two TMA
    // reduce-adds that the dQ warp issues; rows past T are clipped by the
    // tensor map. dqs_free: the previous reduce-adds have read the staging;
    // dqs_full: every softmax warp has written it.
    uint32_t nflush = 0;
    auto flush_dq = [&](uint32_t gg) -> bool {
      uint32_t v[kBwdGradCols];
#pragma unroll
      for (int c16 = 0; c16 < kBwdGradCols; c16 += 16)
        tmem_ld_32x32b_x16(tmem + lane_base + 384 + (gg & 1) * HD + cq * kBwdGradCols + c16,
                           *reinterpret_cast<uint32_t(*)[16]>(v + c16));
      tmem_ld_wait();
      const uint32_t f = nflush++;
      bool fr = mbar_wait(dqs_free, (f & 1) ^ 1u, status, abort_flag, 23);
      if (!__all_sync(0xffffffffu, fr)) return false;
      const int col0 = cq * kBwdGradCols;  // of the 64 dQ columns
      uint8_t* half = sDQ + (col0 >> 5) * TILE_BYTES;
#pragma unroll
      for (int k = 0; k < kBwdGradCols / 4; ++k) {
        const int chunk = ((col0 & 31) >> 2) + k;  // 16-byte chunk of the 128-byte row
        *reinterpret_cast<uint4*>(half + sw128(r, chunk)) = make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(dqs_full);
      return true;
    };
    // dK (scaled) and dV of key tile kt, columns cq*16..+16: TMEM lane = key row.
    // tcgen05.ld is warp-collective (.sync.aligned): every lane loads, only
    // lanes of keys < T store.
    auto drain_dkv = [&](int b, int h, int kt) {
      const int tk = kt * TILE + r;
      const bool key_ok = tk < T;
      // element offset of this key's dK slice; dV is C further
      const long long dk_off =
          (static_cast<long long>(b) * T + (key_ok ? tk : 0)) * 3 * C + C + h * HD + cq * kBwdGradCols;
#pragma unroll
      for (int part = 0; part < 2 * kBwdGradCols / 16; ++part) {  // dK (cols 320.., scaled), then dV (cols 256..)
        const int which = part / (kBwdGradCols / 16), c16 = (part % (kBwdGradCols / 16)) * 16;
        uint32_t x[16];
        tmem_ld_32x32b_x16(tmem + lane_base + (which == 0 ? 320 : 256) + cq * kBwdGradCols + c16, x);
        tmem_ld_wait();
        if (key_ok) {
          const float sc = which == 0 ? 0.125f : 1.0f;
          const long long off = dk_off + (which == 0 ? 0 : C) + c16;
          if (io_f32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(dqkv_ptr) + off);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
              dst[ch] = make_float4(__uint_as_float(x[ch * 4]) * sc, __uint_as_float(x[ch * 4 + 1]) * sc,
                                    __uint_as_float(x[ch * 4 + 2]) * sc, __uint_as_float(x[ch * 4 + 3]) * sc);
          } else {
            uint16_t* dst = static_cast<uint16_t*>(dqkv_ptr) + off;
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
              uint4 u;
              u.x = pack16x2<kF16>(__uint_as_float(x[ch * 8 + 0]) * sc, __uint_as_float(x[ch * 8 + 1]) * sc);
              u.y = pack16x2<kF16>(__uint_as_float(x[ch * 8 + 2]) * sc, __uint_as_float(x[ch * 8 + 3]) * sc);
              u.z = pack16x2<kF16>(__uint_as_float(x[ch * 8 + 4]) * sc, __uint_as_float(x[ch * 8 + 5]) * sc);
              u.w = pack16x2<kF16>(__uint_as_float(x[ch * 8 + 6]) * sc, __uint_as_float(x[ch * 8 + 7]) * sc);
              reinterpret_cast<uint4*>(dst)[ch] = u;
            }
          }
        }
      }
    };
    bool ok = true;
    uint32_t g = 0;
    int stage = 0;
    uint32_t phase = 0;
    bool have_prev = false, prev_last = false;
    int pbb = 0, phh = 0, pkt = 0;  // the previous step's batch, head and key tile
    // the previous step's gradient MMAs are done: flush its dQ and, at an item
    // boundary, drain its item's dK / dV
    auto finish_prev = [&]() -> bool {
      const uint32_t gp = g - 1;
      bool gd = mbar_wait(grad_done + (gp & 1), (gp >> 1) & 1, status, abort_flag, 17);
      if (!__all_sync(0xffffffffu, gd)) return false;
      tc_fence_after();
      if (!flush_dq(gp)) return false;
      if (prev_last) drain_dkv(pbb, phh, pkt);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dq_free + (gp & 1));
        if (prev_last) mbar_arrive(dkv_free);
      }
      return true;
    };
    for (int w = slot(0), nw = 0; w < n_items && ok; w = slot(++nw)) {
      const AttnItem it = bwd_item(w, B, NH);
      const int kt = it.tile, nqi = nk - kt, k0 = kt * TILE;
      for (int j = 0; j < nqi; ++j, ++g) {
        const int qt = kt + j;
        const uint32_t pb = g & 1;
        bool wt = mbar_wait(ld_full + stage, phase, status, abort_flag, 15) &&
                  mbar_wait(sdp_full, g & 1, status, abort_flag, 16);
        if (!__all_sync(0xffffffffu, wt)) { ok = false; break; }
        tc_fence_after();
        // this warp's key columns of S and dP into registers, then release the TMEM
        uint32_t sv[kBwdCols], dv[kBwdCols];
#pragma unroll
        for (int h32 = 0; h32 < kBwdCols / 32; ++h32) {
          tmem_ld_32x32b_x32(tmem + lane_base + cq * kBwdCols + h32 * 32,
                             *reinterpret_cast<uint32_t(*)[32]>(sv + h32 * 32));
          tmem_ld_32x32b_x32(tmem + lane_base + 128 + cq * kBwdCols + h32 * 32,
                             *reinterpret_cast<uint32_t(*)[32]>(dv + h32 * 32));
        }
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sdp_free);
        // P / dS of this warp's key columns, packed in registers
        const float* ld = sLD + stage * 2 * TILE;
        const float nl2 = ld[r] * -kLog2e, drow = ld[TILE + r];
        const int tk0 = k0 + cq * kBwdCols, tq = qt * TILE + r;
        uint32_t pk[kBwdCols / 2], dk[kBwdCols / 2];
        if (qt == kt || qt * TILE + TILE > T)
          bwd_p_ds<true, kBwdCols, kF16>(sv, dv, nl2, drow, tk0, tq, T, pk, dk);
        else
          bwd_p_ds<false, kBwdCols, kF16>(sv, dv, nl2, drow, tk0, tq, T, pk, dk);
        // the single P / dS buffer: the previous step's gradient MMAs have read it
        if (have_prev) {
          const uint32_t gp = g - 1;
          bool gd = mbar_wait(grad_done + (gp & 1), (gp >> 1) & 1, status, abort_flag, 17);
          if (!__all_sync(0xffffffffu, gd)) { ok = false; break; }
          tc_fence_after();
        }
#pragma unroll
        for (int c = 0; c < kBwdCols / 8; ++c) {
          const int chunk = cq * kBwdCols / 8 + c;
          const uint32_t off = (chunk >> 3) * TILE_BYTES + sw128(r, chunk & 7);
          *reinterpret_cast<uint4*>(sPD + off) = make_uint4(pk[c * 4], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
          *reinterpret_cast<uint4*>(sPD + 2 * TILE_BYTES + off) =
              make_uint4(dk[c * 4], dk[c * 4 + 1], dk[c * 4 + 2], dk[c * 4 + 3]);
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ps_full + pb);
        if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        if (have_prev && !finish_prev()) { ok = false; break; }
        have_prev = true;
        prev_last = j + 1 == nqi;
        pbb = it.b;
        phh = it.h;
        pkt = kt;
      }
    }
    if (ok && have_prev) finish_prev();
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Raises a kernel's dynamic shared memory limit once per (kernel, device).
int set_smem(const void* k, size_t bytes) {
  static const void* kernels[8] = {};
  static bool done[8][64] = {};
  int dev = 0;
  LLMK_CUDA(cudaGetDevice(&dev));
  int slot = 0;
  while (slot < 8 && kernels[slot] && kernels[slot] != k) ++slot;
  if (slot == 8 || dev >= 64) {
    LLMK_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
    return LLMK_OK;
  }
  kernels[slot] = k;
  if (!done[slot][dev]) {
    LLMK_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
    done[slot][dev] = true;
  }
  return LLMK_OK;
}

// The last, partial round of the snake schedule (sched_slot_tail): ranks the
// CTAs by the work the full rounds gave them, least first, ties by CTA index.
// An item's work is its key-tile steps plus one for its set-up: forward pair
// item p (2p+1 and 2p+2 key tiles), backward key tile kt (nq - kt query tiles).
void attn_sched_tail(bool bwd, int n_items, int g, int nq, int bh_count, SchedTail& t) {
  thread_local int key[5] = {-1, -1, -1, -1, -1};
  thread_local SchedTail cached;
  if (key[0] == static_cast<int>(bwd) && key[1] == n_items && key[2] == g && key[3] == nq && key[4] == bh_count) {
    t = cached;
    return;
  }
  const int np = (nq + 1) / 2, full = n_items / g, rem = n_items - full * g;
  std::vector<long long> load(g, 0);
  std::vector<int> order(g);
  for (int c = 0; c < g; ++c) {
    order[c] = c;
    for (int k = 0; k < full; ++k) {
      const int w = k * g + ((k & 1) ? g - 1 - c : c);
      if (bwd) {
        load[c] += nq - w / bh_count + 1;
      } else {
        const int p = np - 1 - w / bh_count;
        load[c] += (2 * p + 1) + (2 * p + 1 < nq ? 2 * p + 2 : 0) + 1;
      }
    }
  }
  std::sort(order.begin(), order.end(), [&](int a, int b) { return load[a] != load[b] ? load[a] < load[b] : a < b; });
  for (int c = 0; c < kMaxTailCtas; ++c) t.slot[c] = -1;
  for (int r = 0; r < rem; ++r) t.slot[order[r]] = static_cast<int16_t>(r);
  key[0] = static_cast<int>(bwd); key[1] = n_items; key[2] = g; key[3] = nq; key[4] = bh_count;
  cached = t;
}

int check_shapes(int B, int T, int C3, int NH) {
  if (B <= 0 || T <= 0 || C3 <= 0 || NH <= 0 || C3 % 3) return fail(LLMK_ERR_INVALID_ARG, "attention: bad shape");
  const int C = C3 / 3;
  if (C % NH || C / NH != HD) return fail(LLMK_ERR_UNSUPPORTED, "attention: head size must be 64");
  return LLMK_OK;
}

}  // namespace
}  // namespace llmk

using namespace llmk;

extern "C" {

int llmk_attention_forward(void* out, llmk_dtype out_dtype, float* lse, const void* qkv, llmk_dtype qkv_dtype, int B,
                           int T, int C3, int NH, void* stream) {
  if (!out || !lse || !qkv) return fail(LLMK_ERR_INVALID_ARG, "attention_forward: null pointer");
  LLMK_TRY(check_shapes(B, T, C3, NH));
  if (qkv_dtype != LLMK_BF16 && qkv_dtype != LLMK_F16)
    return fail(LLMK_ERR_UNSUPPORTED, "attention_forward: qkv dtype (bf16 or fp16)");
  if (out_dtype != qkv_dtype && out_dtype != LLMK_F32)
    return fail(LLMK_ERR_UNSUPPORTED, "attention_forward: out dtype (qkv's or fp32)");
  if (!aligned16(out) || !aligned16(qkv)) return fail(LLMK_ERR_UNSUPPORTED, "attention_forward: alignment");
  const bool f16 = qkv_dtype == LLMK_F16;
  const int C = C3 / 3;
  CUtensorMap tm;
  LLMK_TRY(make_tmap_3d(&tm, qkv, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C3, T, B,
                        static_cast<uint64_t>(C3) * 2, static_cast<uint64_t>(T) * C3 * 2, HD, TILE, 1));
  auto kern = f16 ? attn_fwd_kernel<true> : attn_fwd_kernel<false>;
  LLMK_TRY(set_smem(reinterpret_cast<const void*>(kern), FwdSmem::BYTES));
  const int nq = (T + TILE - 1) / TILE;
  const int np = (nq + 1) / 2;  // pairs of query tiles
  // persistent: one CTA per SM
  const int grid = std::min(std::min(np * B * NH, num_sms()), kMaxTailCtas);
  SchedTail tail;
  attn_sched_tail(false, np * B * NH, grid, nq, B * NH, tail);
  kern<<<grid, kFwdThreads, FwdSmem::BYTES, static_cast<cudaStream_t>(stream)>>>(
      tm, out, out_dtype == LLMK_F32 ? 1 : 0, lse, B, T, NH, C, device_status_ptr(), tail);
  count_launch();
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

static size_t attn_ws_parts(int B, int T, int C, int NH, size_t* dq_off, size_t* do16_off) {
  const size_t d = ((static_cast<size_t>(B) * NH * T * sizeof(float) + 255) / 256) * 256;
  const size_t dq = ((static_cast<size_t>(B) * T * C * sizeof(float) + 255) / 256) * 256;
  const size_t do16 = static_cast<size_t>(B) * T * C * 2;
  if (dq_off) *dq_off = d;
  if (do16_off) *do16_off = d + dq;
  return d + dq + do16;
}

size_t llmk_attention_backward_workspace(int B, int T, int C3, int NH) {
  if (B <= 0 || T <= 0 || C3 <= 0 || NH <= 0) return 0;
  return attn_ws_parts(B, T, C3 / 3, NH, nullptr, nullptr);
}

}  // extern "C"

namespace {

template <bool kF16>
int attention_backward_t(void* dqkv, const void* dout, const void* out, bool f32, const void* qkv, const float* lse,
                         int B, int T, int C3, int NH, void* workspace, cudaStream_t s) {
  using T16 = typename std::conditional<kF16, __half, __nv_bfloat16>::type;
  const int C = C3 / 3;
  size_t dq_off, do16_off;
  attn_ws_parts(B, T, C, NH, &dq_off, &do16_off);
  float* Dv = static_cast<float*>(workspace);
  float* dq = reinterpret_cast<float*>(static_cast<char*>(workspace) + dq_off);
  uint16_t* do16 = reinterpret_cast<uint16_t*>(static_cast<char*>(workspace) + do16_off);
  const long long rows = static_cast<long long>(B) * T;  // one warp per (b, t)
  const int pre_grid = static_cast<int>((rows + 7) / 8);
  if (f32)
    attn_bwd_pre_kernel<float, kF16><<<pre_grid, 256, 0, s>>>(Dv, dq, do16, static_cast<const float*>(dout),
                                                              static_cast<const float*>(out), B, T, NH, C);
  else
    attn_bwd_pre_kernel<T16, kF16><<<pre_grid, 256, 0, s>>>(Dv, dq, nullptr, static_cast<const T16*>(dout),
                                                            static_cast<const T16*>(out), B, T, NH, C);
  // the MMAs read dO in the operand type: the caller's buffer, or the copy the pre-pass made
  const void* dout_mma = f32 ? static_cast<const void*>(do16) : dout;
  const CUtensorMapDataType dt = kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, td;
  LLMK_TRY(make_tmap_3d(&tq, qkv, dt, C3, T, B, static_cast<uint64_t>(C3) * 2, static_cast<uint64_t>(T) * C3 * 2, HD,
                        TILE, 1));
  LLMK_TRY(make_tmap_3d(&td, dout_mma, dt, C, T, B, static_cast<uint64_t>(C) * 2, static_cast<uint64_t>(T) * C * 2, HD,
                        TILE, 1));
  CUtensorMap tdq;  // fp32 dQ accumulator (B, T, C), [128 x 32] boxes for the reduce-adds
  LLMK_TRY(make_tmap_3d(&tdq, dq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, C, T, B, static_cast<uint64_t>(C) * 4,
                        static_cast<uint64_t>(T) * C * 4, 32, TILE, 1));
  LLMK_TRY(set_smem(reinterpret_cast<const void*>(attn_bwd_kernel<kF16>), BwdSmem::BYTES));
  const int nk = (T + TILE - 1) / TILE;
  // persistent: one CTA per SM walking key-tile items in the snake-order
  // schedule, so an item's dK / dV drain and K / V load overlap the next
  // item's first query tile
  const int grid = std::min(std::min(nk * B * NH, num_sms()), kMaxTailCtas);
  SchedTail tail;
  attn_sched_tail(true, nk * B * NH, grid, nk, B * NH, tail);
  attn_bwd_kernel<kF16><<<grid, kBwdThreads, BwdSmem::BYTES, s>>>(tq, td, tdq, dqkv, f32 ? 1 : 0, dq, lse, Dv, B, T, NH, C,
                                                                  device_status_ptr(), tail);
  const long long n8 = static_cast<long long>(B) * T * C / 8;
  const int pg = static_cast<int>(std::min<long long>((n8 + 255) / 256, 148LL * 16));
  if (f32) attn_bwd_post_kernel<float, kF16><<<pg, 256, 0, s>>>(static_cast<float*>(dqkv), dq, B * T, C, 0.125f);
  else attn_bwd_post_kernel<T16, kF16><<<pg, 256, 0, s>>>(static_cast<T16*>(dqkv), dq, B * T, C, 0.125f);
  count_launch(3);
  LLMK_CUDA(cudaGetLastError());
  return LLMK_OK;
}

}  // namespace

extern "C" {

int llmk_attention_backward(void* dqkv, const void* dout, const void* out, llmk_dtype io_dtype, const void* qkv,
                            llmk_dtype qkv_dtype, const float* lse, int B, int T, int C3, int NH, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!dqkv || !dout || !out || !qkv || !lse) return fail(LLMK_ERR_INVALID_ARG, "attention_backward: null pointer");
  LLMK_TRY(check_shapes(B, T, C3, NH));
  if (qkv_dtype != LLMK_BF16 && qkv_dtype != LLMK_F16)
    return fail(LLMK_ERR_UNSUPPORTED, "attention_backward: qkv dtype (bf16 or fp16)");
  if (io_dtype != qkv_dtype && io_dtype != LLMK_F32)
    return fail(LLMK_ERR_UNSUPPORTED, "attention_backward: io dtype (qkv's or fp32)");
  if (!aligned16(dqkv) || !aligned16(dout) || !aligned16(out) || !aligned16(qkv))
    return fail(LLMK_ERR_UNSUPPORTED, "attention_backward: alignment");
  if (!workspace || workspace_bytes < llmk_attention_backward_workspace(B, T, C3, NH) || !aligned16(workspace))
    return fail(LLMK_ERR_WORKSPACE, "attention_backward: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f32 = io_dtype == LLMK_F32;
  if (qkv_dtype == LLMK_F16) return attention_backward_t<true>(dqkv, dout, out, f32, qkv, lse, B, T, C3, NH, workspace, s);
  return attention_backward_t<false>(dqkv, dout, out, f32, qkv, lse, B, T, C3, NH, workspace, s);
}

}  // extern "C"
