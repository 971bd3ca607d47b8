// gemv.cu -- the grouped expert products for small batches (4 < T <= 64)
// as bandwidth-bound batched GEMVs.
//
// Reference behaviour: the decode-regime phases moe_phase1_gate_up_act and
// moe_phase2_down (Sources/Tsugumi/Metal/MoE/moe.metal:455-574, :651-687;
// MoE.swift:529-644) -- per routed slot, act = act_fn(gate . x) * (up . x),
// then down . act -- over the token rows the prefill front end has already
// routed, grouped by expert and gathered (normalised fp16 rows in expert
// order, shared-expert rows appended: the row tiles of the schedule).  They
// replace the two tcgen05 contraction launches when every expert holds few
// tokens: the tensor-core path pays a fixed cost per 128 weight rows that
// only wide tiles amortise, while here the cost is the weight bytes.
//
// One warp per work item; each lane owns whole 32-element groups of int4
// codes (group 4 s + c of a 4-group super-group: int4_mma.cuh), dequantises
// them in registers and multiplies them with mma.sync m16n8k16 against the
// tile's token rows (8 tokens per MMA column block, up to 8 blocks; the rows
// are read through L1, stored in MMA fragment order -- each 8 elements as
// x0 x4 x2 x6 x1 x5 x3 x7 -- by the gather kernel and by the gate/up pass):
//   gate/up  item = (row tile, 8 f): MMA rows 0-7 are the gate rows, 8-15
//            the up rows of the same f, so a lane holds gate and up of its
//            (f, token) pair and writes act = act_fn(g) * u as fp16;
//   down     item = (row tile, 16 output rows d): partials[row][d] in fp16,
//            which the combine kernel reads as for the tensor-core path.
// To cover DRAM latency each warp keeps kStages super-groups of codes and
// scales in flight: cp.async copies (16 bytes of codes per lane and row, 4
// bytes of scales) into a ring in shared memory that only the copying lane
// reads back, issued kStages - 1 steps ahead across item boundaries.  With
// that, instruction issue bounds the kernel (~200 instructions per warp and
// KB of codes, 96 of them the exact dequantisation), not the weight stream.
// A CTA takes a contiguous range of items, so its warps mostly share a row
// tile and read its token rows from L1.
#include "int4_mma.cuh"
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kMaxBlk = 8;  // token column blocks of 8: up to 64 rows per tile
// one ring slot: codes of rows a (lane * 16) and b (512 + lane * 16), then
// the scales, 16 bytes per row pair g: a's four groups, b's four groups
constexpr int kSlotBytes = 1024 + 128;

// Launch shape by the largest tile (MAXB token blocks): 16 warps per CTA
// (measured: 576 or 640 threads were slower, and 576 spilled at B = 2); one
// token block leaves registers for two accumulator chains (the MMAs of a
// super-group alternate between them).
template <int MAXB>
struct GemvShape {
  static constexpr int kThreads = 512;
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kStages = MAXB <= 2 ? 6 : 8;  // super-groups in flight per warp
  static constexpr int kChains = MAXB == 1 ? 2 : 1;
  static constexpr int kWarpRing = kStages * kSlotBytes;
  static constexpr size_t kSmem = static_cast<size_t>(kWarps) * kWarpRing;
};

struct GemvArgs {
  const uint8_t* ebase;
  uint64_t estride;
  ExpertOffsets off;
  const uint8_t* shared;
  ExpertOffsets soff;
  const RowTile* tiles;
  const uint32_t* n_tiles;
  int D, F, E, act;
  const __half* xp;   // [rows][D]
  __half* act_buf;    // [rows][F]
  __half* partials;   // [rows][D]
  uint32_t* err;
};

// cp.async of 16 / 4 bytes to shared address dst + OFF; the "z" forms copy
// `n` source bytes (0 or the full size) and zero-fill the rest.
template <int OFF>
TSG_DEV void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0+%2], [%1], 16;" ::"r"(dst), "l"(src), "n"(OFF)
               : "memory");
}
template <int OFF>
TSG_DEV void cp16z(uint32_t dst, const void* src, uint32_t n) {
  asm volatile("cp.async.cg.shared.global [%0+%3], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n),
               "n"(OFF)
               : "memory");
}
TSG_DEV void cp4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
TSG_DEV void cp4z(uint32_t dst, const void* src, uint32_t n) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
TSG_DEV uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
TSG_DEV uint4 lds128_512(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+512];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
TSG_DEV void lds_scale_pair(uint32_t addr, __half* a, __half* b) {
  unsigned short x, y;
  asm volatile("ld.shared.u16 %0, [%2];\n\tld.shared.u16 %1, [%2+8];" : "=h"(x), "=h"(y) : "r"(addr));
  *a = __ushort_as_half(x);
  *b = __ushort_as_half(y);
}
TSG_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
TSG_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The row tiles of a CTA's item range, staged in shared memory at the start
// (an item switch then costs no global-memory round trip); ranges over more
// tiles than the cache holds read the rest from global memory.
constexpr int kTileCache = 32;
struct TileCache {
  const RowTile* s;  // shared memory
  uint32_t t0, n;
  TSG_DEV RowTile get(const GemvArgs& a, uint32_t t) const {
    return t - t0 < n ? s[t - t0] : a.tiles[t];
  }
};

// The producer's copy cursor for one item: the lane's code group 4 s + c of
// weight rows a = g and b = g + 8 of the item's 16-row MMA block, its scale
// pair (groups 4 s + (c & 2), + 1; of row a for even c, of row b for odd c)
// and the groups left in the row from group 4 s on.
struct Cursor {
  const uint8_t* ca;
  const uint8_t* cb;
  const __half* sc;
  int left;
};

template <int MODE>
TSG_DEV Cursor item_cursor(const GemvArgs& a, const TileCache& tc, uint32_t item, int per_tile,
                           int g, int c, int ngroups) {
  const uint32_t t = item / static_cast<uint32_t>(per_tile);
  const int sub = static_cast<int>(item - t * static_cast<uint32_t>(per_tile));
  const uint32_t expert = tc.get(a, t).expert;
  const bool sh = expert >= static_cast<uint32_t>(a.E);
  const ExpertOffsets& o = sh ? a.soff : a.off;
  const uint8_t* blob = sh ? a.shared : a.ebase + static_cast<uint64_t>(expert) * a.estride;
  const uint8_t *ca, *cb;
  const __half *sa, *sb;
  if (MODE == 0) {
    const size_t f = static_cast<size_t>(sub) * 8 + g;
    ca = blob + o.gate_w + f * (a.D / 2);
    cb = blob + o.up_w + f * (a.D / 2);
    sa = reinterpret_cast<const __half*>(blob + o.gate_s) + f * (a.D / 32);
    sb = reinterpret_cast<const __half*>(blob + o.up_s) + f * (a.D / 32);
  } else {
    const size_t d = static_cast<size_t>(sub) * 16 + g;
    ca = blob + o.down_w + d * (a.F / 2);
    cb = blob + o.down_w + (d + 8) * (a.F / 2);
    sa = reinterpret_cast<const __half*>(blob + o.down_s) + d * (a.F / 32);
    sb = reinterpret_cast<const __half*>(blob + o.down_s) + (d + 8) * (a.F / 32);
  }
  Cursor r;
  r.ca = ca + c * 16;
  r.cb = cb + c * 16;
  r.sc = ((c & 1) ? sb : sa) + (c & 2);
  r.left = ngroups;
  return r;
}

// Copies the cursor's super-group into a ring slot (codes of rows a and b at
// lane * 16 and 512 + lane * 16; scales at 1024 + g * 16: a's four groups,
// then b's) and advances it.  `dst` is the slot + lane * 16, `sdst` the
// lane's scale destination.  Groups past the row end (an even count) are
// zero-filled from a valid address in the row: a zero scale and zero tokens
// make them contribute nothing.
TSG_DEV void issue_step(uint32_t dst, uint32_t sdst, Cursor& r, int c) {
  if (r.left >= 4) {  // warp-uniform: a whole super-group
    cp16<0>(dst, r.ca);
    cp16<512>(dst, r.cb);
    cp4(sdst, r.sc);
  } else {
    const bool okc = c < r.left;
    const bool oks = (c & 2) < r.left;
    cp16z<0>(dst, okc ? r.ca : r.ca - 16 * c, okc ? 16u : 0u);
    cp16z<512>(dst, okc ? r.cb : r.cb - 16 * c, okc ? 16u : 0u);
    cp4z(sdst, oks ? r.sc : r.sc - (c & 2), oks ? 4u : 0u);
  }
  r.ca += 64;
  r.cb += 64;
  r.sc += 4;
  r.left -= 4;
}

// One super-group of two weight-row halves (rows g and g + 8 of the MMA)
// against nblk token blocks.  `ra` / `rb` are the lane's 16 code bytes of
// its group in the two rows, sa / sb their fp16 scales (with s / 16);
// `bgrp` points at the group in the lane's token row of block 0 (token g),
// stored in MMA fragment order (int4_mma.cuh), block tb being `blk_stride`
// further each.  The lane's row exists in blocks below `nb_lane`; elsewhere
// it reads the tile's first row instead (`absent` back from bgrp): the MMA
// column of a missing token is never stored.  Past the end of the row the
// caller points bgrp at a group inside it: the zero-filled weights make
// those products zero.
template <int MAXB, int CH>
TSG_DEV void super_group(float (&acc)[MAXB][CH][4], const uint4& ra, const uint4& rb, __half2 sa,
                         __half2 sa16, __half2 sb, __half2 sb16, const __half* bgrp,
                         size_t blk_stride, ptrdiff_t absent, int nb_lane, int nblk) {
  const uint32_t wa[4] = {ra.x, ra.y, ra.z, ra.w};
  const uint32_t wb[4] = {rb.x, rb.y, rb.z, rb.w};
  uint32_t pa[4][4], pb[4][4];
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    dequant_word(wa[wi], sa, sa16, pa[wi]);
    dequant_word(wb[wi], sb, sb16, pb[wi]);
  }
#pragma unroll
  for (int tb = 0; tb < MAXB; ++tb) {
    if (tb >= nblk) break;
    uint4 bx[4];
    const uint4* src = reinterpret_cast<const uint4*>(
        bgrp + (tb < nb_lane ? static_cast<ptrdiff_t>(tb * blk_stride) : absent));
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) bx[wi] = __ldg(src + wi);
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      float(&d)[4] = acc[tb][wi % CH];
      mma_16816(d, pa[wi][0], pb[wi][0], pa[wi][1], pb[wi][1], bx[wi].x, bx[wi].y);
      mma_16816(d, pa[wi][2], pb[wi][2], pa[wi][3], pb[wi][3], bx[wi].z, bx[wi].w);
    }
  }
}

TSG_DEV void split_scale(__half s, __half2* s2, __half2* s16) {
  *s2 = __halves2half2(s, s);
  *s16 = __hmul2(*s2, bits_h2(0x2C002C00u));  // (s / 16, s / 16), exact
}

template <int MODE, int ACT, int MAXB>
__global__ void __launch_bounds__(GemvShape<MAXB>::kThreads, 1) gemv_kernel(const GemvArgs a) {
  using S = GemvShape<MAXB>;
  constexpr int kWarps = S::kWarps, kStages = S::kStages, CH = S::kChains;
  extern __shared__ __align__(16) uint8_t gemv_smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const uint32_t n_tiles = __ldg(a.n_tiles);
  // rows per item: 8 f (gate + up) or 16 d
  const int K = MODE == 0 ? a.D : a.F;
  const int per_tile = MODE == 0 ? a.F / 8 : a.D / 16;
  const int ngroups = K / 32;
  const int nsg = (ngroups + 3) / 4;
  const uint32_t n_items = n_tiles * static_cast<uint32_t>(per_tile);
  // this CTA's contiguous item range; its warps stride through it
  const uint32_t lo = static_cast<uint32_t>(
      static_cast<uint64_t>(n_items) * blockIdx.x / gridDim.x);
  const uint32_t hi = static_cast<uint32_t>(
      static_cast<uint64_t>(n_items) * (blockIdx.x + 1) / gridDim.x);
  const __half* bsrc = MODE == 0 ? a.xp : a.act_buf;
  __shared__ RowTile s_tiles[kTileCache];
  TileCache tc;
  tc.s = s_tiles;
  tc.t0 = lo / static_cast<uint32_t>(per_tile);
  tc.n = hi > lo ? (hi - 1) / static_cast<uint32_t>(per_tile) - tc.t0 + 1 : 0u;
  if (tc.n > static_cast<uint32_t>(kTileCache)) tc.n = kTileCache;
  if (threadIdx.x < tc.n) s_tiles[threadIdx.x] = a.tiles[tc.t0 + threadIdx.x];
  __syncthreads();
  // the lane's addresses in the warp's ring: slot + lane * 16, advancing by
  // one slot per step and wrapping; scale destination and source offsets
  const uint32_t ring_lane =
      static_cast<uint32_t>(__cvta_generic_to_shared(gemv_smem + warp * S::kWarpRing)) + lane * 16;
  const uint32_t ring_end = ring_lane + kStages * kSlotBytes;
  const uint32_t s_put = 1024 + g * 16 + (c & 1) * 8 + (c & 2) * 2 - lane * 16;
  const uint32_t s_get = 1024 + g * 16 + c * 2 - lane * 16;

  // producer cursor: runs kStages - 1 steps ahead of the consumer
  uint32_t p_item = lo + warp;
  uint32_t p_slot = ring_lane;
  Cursor pr{};
  if (p_item < hi) pr = item_cursor<MODE>(a, tc, p_item, per_tile, g, c, ngroups);
  auto produce = [&]() {
    if (p_item < hi) {
      issue_step(p_slot, p_slot + s_put, pr, c);
      if (pr.left <= 0) {
        p_item += kWarps;
        if (p_item < hi) pr = item_cursor<MODE>(a, tc, p_item, per_tile, g, c, ngroups);
      }
    }
    cp_async_commit();  // an empty group keeps the count uniform
    p_slot += kSlotBytes;
    if (p_slot == ring_end) p_slot = ring_lane;
  };
#pragma unroll 1
  for (int i = 0; i < kStages - 1; ++i) produce();

  uint32_t c_slot = ring_lane;
  for (uint32_t item = lo + warp; item < hi; item += kWarps) {
    const uint32_t t = item / static_cast<uint32_t>(per_tile);
    const int sub = static_cast<int>(item - t * static_cast<uint32_t>(per_tile));
    const RowTile tile = tc.get(a, t);
    const bool bad = static_cast<int>(tile.rows) > 8 * MAXB;
    if (bad && lane == 0) flag_error(a.err, TSG_DEVERR_BOUNDS);  // the host keeps tiles <= 64 rows
    const int cnt = bad ? 0 : static_cast<int>(tile.rows);
    const int nblk = (cnt + 7) / 8;
    const int nb_lane = cnt > g ? (cnt - g + 7) / 8 : 0;
    // the lane's group in its token row of block 0 (token g); block tb is
    // 8 rows further
    const __half* bp = bsrc + static_cast<size_t>(tile.row_start + g) * K + c * 32;
    const size_t blk_stride = static_cast<size_t>(8) * K;
    const ptrdiff_t absent = -static_cast<ptrdiff_t>(g) * K;  // back to the tile's first row
    float acc[MAXB][CH][4];
#pragma unroll
    for (int tb = 0; tb < MAXB; ++tb)
#pragma unroll
      for (int ch = 0; ch < CH; ++ch) acc[tb][ch][0] = acc[tb][ch][1] = acc[tb][ch][2] = acc[tb][ch][3] = 0.0f;

#pragma unroll 1
    for (int s = 0; s < nsg; ++s) {
      produce();
      cp_async_wait<kStages - 1>();  // this step's slot has landed
      const uint4 ra = lds128(c_slot);
      const uint4 rb = lds128_512(c_slot);
      __half sa, sb;
      lds_scale_pair(c_slot + s_get, &sa, &sb);
      c_slot += kSlotBytes;
      if (c_slot == ring_end) c_slot = ring_lane;
      __half2 sa2, sa16, sb2, sb16;
      split_scale(sa, &sa2, &sa16);
      split_scale(sb, &sb2, &sb16);
      super_group<MAXB, CH>(acc, ra, rb, sa2, sa16, sb2, sb16,
                            4 * s + c < ngroups ? bp : bp - c * 32, blk_stride, absent, nb_lane,
                            nblk);
      bp += 128;
    }

    // lane (g, c): acc[tb][.][0..1] = row g for tokens 2c, 2c+1; [2..3] = row g + 8
#pragma unroll
    for (int tb = 0; tb < MAXB; ++tb) {
      if (tb >= nblk) break;
#pragma unroll
      for (int ch = 1; ch < CH; ++ch)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[tb][0][i] += acc[tb][ch][i];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = tb * 8 + 2 * c + h;
        if (n >= cnt) continue;
        const size_t row = tile.row_start + static_cast<size_t>(n);
        if (MODE == 0) {
          // act rows in MMA fragment order for the down pass: element j of
          // each 8 at ((j & 1) << 2) | (j & 2) | (j >> 2)
          const int f = sub * 8 + (((g & 1) << 2) | (g & 2) | (g >> 2));
          a.act_buf[row * a.F + f] =
              __float2half_rn(gate_act_fast(ACT, acc[tb][0][h]) * acc[tb][0][2 + h]);
        } else {
          const int d = sub * 16 + g;
          a.partials[row * a.D + d] = __float2half_rn(acc[tb][0][h]);
          a.partials[row * a.D + d + 8] = __float2half_rn(acc[tb][0][2 + h]);
        }
      }
    }
  }
  cp_async_wait<0>();
}

GemvArgs gemv_args(const QmmParams& p) {
  GemvArgs a;
  a.ebase = p.experts.base;
  a.estride = p.experts.stride;
  a.off = p.experts.off;
  a.shared = p.experts.shared;
  a.soff = p.experts.shared_off;
  a.tiles = p.row_tiles;
  a.n_tiles = p.n_row_tiles;
  a.D = p.D;
  a.F = p.F;
  a.E = p.E;
  a.act = p.act;
  a.xp = p.xp;
  a.act_buf = p.act_buf;
  a.partials = p.partials;
  a.err = p.err;
  return a;
}

}  // namespace

int gemv_max_tile_rows() { return 8 * kMaxBlk; }

bool gemv_usable(const QmmParams& p) {
  // whole super-groups of gate/up rows; an even group count and 4-byte
  // aligned scale planes for the 4-byte scale copies; 16-byte aligned code
  // planes for the 16-byte code copies
  const ExpertOffsets& o = p.experts.off;
  const ExpertOffsets& so = p.experts.shared_off;
  const uint32_t blobs = static_cast<uint32_t>(p.experts.stride) |
                         static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.experts.base)) |
                         static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.experts.shared));
  const uint32_t codes = o.gate_w | o.up_w | o.down_w | so.gate_w | so.up_w | so.down_w | blobs;
  const uint32_t scales = o.gate_s | o.up_s | o.down_s | so.gate_s | so.up_s | so.down_s | blobs;
  return p.D % 128 == 0 && p.F % 64 == 0 && (codes & 15u) == 0 && (scales & 3u) == 0;
}

namespace {
template <int MODE, int ACT, int MAXB>
cudaError_t launch_shape(const QmmParams& p, cudaStream_t s) {
  using S = GemvShape<MAXB>;
  cudaError_t e = allow_max_smem(gemv_kernel<MODE, ACT, MAXB>);
  if (e != cudaSuccess) return e;
  gemv_kernel<MODE, ACT, MAXB><<<p.num_sms, S::kThreads, S::kSmem, s>>>(gemv_args(p));
  return cudaGetLastError();
}
template <int MODE, int ACT>
cudaError_t launch_mode(const QmmParams& p, int max_rows, cudaStream_t s) {
  if (!gemv_usable(p) || max_rows < 1 || max_rows > 8 * kMaxBlk) return cudaErrorInvalidValue;
  if (max_rows <= 8) return launch_shape<MODE, ACT, 1>(p, s);
  if (max_rows <= 16) return launch_shape<MODE, ACT, 2>(p, s);
  if (max_rows <= 32) return launch_shape<MODE, ACT, 4>(p, s);
  return launch_shape<MODE, ACT, 8>(p, s);
}
}  // namespace

cudaError_t launch_gemv_gate_up(const QmmParams& p, int max_rows, cudaStream_t s) {
  return p.act == 1 ? launch_mode<0, 1>(p, max_rows, s) : launch_mode<0, 0>(p, max_rows, s);
}

cudaError_t launch_gemv_down(const QmmParams& p, int max_rows, cudaStream_t s) {
  return launch_mode<1, 0>(p, max_rows, s);
}

}  // namespace tsg
