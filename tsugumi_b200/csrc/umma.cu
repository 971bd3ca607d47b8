// umma.cu -- the prefill-regime grouped int4 contraction on tcgen05.
//
// Reference behaviour: prefill_moe_gemm_int4 / _nax
// (Sources/Tsugumi/Metal/Prefill/prefill.metal:893-1075, :3664-3866) driven by
// PrefillGroupedRoutedMoE.encodeStreamedTiled
// (Sources/Tsugumi/Kernels/Prefill/MoE/PrefillGroupedRoutedMoE.swift:931-1051):
// per block of one expert's rows, mode 0 computes the gate and up products of
// the gathered rows and (prefill_moe_gate_up_gelu_mul, prefill.metal:1081-1092)
// act = half(act_fn(gate) * up); mode 1 computes the down product into
// per-route partials.  Weights are dequantised once to fp16 and multiplied
// with fp32 accumulation.
//
// B200 design (one persistent CTA per SM, warp-specialised):
//   * the tensor-core M operand is 128 weight rows (mode 0: 64 gate rows and
//     the 64 matching up rows, so one accumulator tile holds both halves of
//     act; mode 1: 128 down rows); the N operand is the row tile of sorted
//     token rows (<= 128, any multiple of 16), so a lightly routed expert
//     costs only the rows it has;
//   * warps 6-13 dequantise int4 codes (prefetched from global into registers
//     several k-steps ahead) to fp16 straight into the 128-byte-swizzled
//     K-major layout the UMMA descriptor reads;
//   * warp 4 moves token tiles with TMA (tensor maps, no multicast);
//   * warp 5 allocates TMEM and issues tcgen05.mma (M=128, N=rows, K=16) into
//     one of two fp32 accumulator buffers, committing to mbarriers;
//   * warps 0-3 (one per TMEM lane quarter) drain the accumulator with
//     tcgen05.ld, apply the activation or convert, and store fp16 rows.
// Every wait is bounded (tsg_common.cuh) so a fault in the pipeline ends the
// kernel with an error flag instead of hanging the GPU.
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kStagesQ = 5;
constexpr int kTileN = 128;          // max token rows per tile
constexpr int kBoxRows = 16;         // TMA box height (rows)
constexpr int kKStep = 64;           // K per stage (one 128-byte swizzle row)
constexpr int kABytes = 128 * 128;   // 128 weight rows x 64 fp16
constexpr int kBBytes = kTileN * 128;
constexpr int kPrefetch = 4;         // dequant look-ahead in k-steps
constexpr int kThreadsQ = 14 * 32;
constexpr int kDqWarp0 = 6;
constexpr int kNumDqWarps = 8;
constexpr uint32_t kTmemCols = 2 * kTileN;

struct QArgs {
  const uint8_t* ebase;
  uint64_t estride;
  ExpertOffsets off;
  const uint8_t* shared;
  ExpertOffsets soff;
  const RowTile* tiles;
  const uint32_t* n_tiles;
  int K;      // reduction length
  int n_wt;   // weight tiles per row tile
  int E;
  int act;
  int out_cols;  // F (mode 0) or D (mode 1)
  __half* out;
  uint32_t* err;
};

struct SmemQ {
  uint64_t full_a[kStagesQ];
  uint64_t full_b[kStagesQ];
  uint64_t empty[kStagesQ];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  float xchg[64 * 17];  // mode 0: up values handed to the gate warps
};

struct WorkItem {
  uint32_t expert, row_start, rows, wt;
  bool valid;
};

TSG_DEV WorkItem work_item(const QArgs& a, uint32_t n_items, uint32_t idx) {
  WorkItem w;
  w.valid = idx < n_items;
  if (!w.valid) return w;
  const uint32_t rt = idx / static_cast<uint32_t>(a.n_wt);
  w.wt = idx % static_cast<uint32_t>(a.n_wt);
  const RowTile t = a.tiles[rt];
  w.expert = t.expert;
  w.row_start = t.row_start;
  w.rows = t.rows;
  return w;
}

// Source of one dequant thread's 16 code bytes and its fp16 scale for a
// given (item, k-step).
template <int MODE>
TSG_DEV void dq_source(const QArgs& a, const WorkItem& w, int m, int h, int ks,
                       const uint4** codes, const __half** scale) {
  const bool sh = w.expert >= static_cast<uint32_t>(a.E);
  const uint8_t* blob = sh ? a.shared : a.ebase + static_cast<uint64_t>(w.expert) * a.estride;
  const ExpertOffsets& o = sh ? a.soff : a.off;
  uint32_t wo, so, row;
  if (MODE == 0) {
    const uint32_t f0 = w.wt * 64u;
    if (m < 64) { wo = o.gate_w; so = o.gate_s; row = f0 + m; }
    else { wo = o.up_w; so = o.up_s; row = f0 + (m - 64); }
  } else {
    wo = o.down_w; so = o.down_s; row = w.wt * 128u + m;
  }
  const size_t kb = static_cast<size_t>(a.K / 2);
  *codes = reinterpret_cast<const uint4*>(blob + wo + row * kb + ks * 32 + h * 16);
  *scale = reinterpret_cast<const __half*>(blob + so) + static_cast<size_t>(row) * (a.K / 32) +
           2 * ks + h;
}

template <int MODE>
__global__ void __launch_bounds__(kThreadsQ, 1)
    qmm_kernel(const __grid_constant__ CUtensorMap tmap_b, QArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ SmemQ sm;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - smem_u32(smem_raw));
  // stage s: A at base + s*(kABytes+kBBytes), B right after
  auto stage_a = [&](int s) { return gbase + s * (kABytes + kBBytes); };
  auto stage_b = [&](int s) { return gbase + s * (kABytes + kBBytes) + kABytes; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t n_items = __ldg(a.n_tiles) * static_cast<uint32_t>(a.n_wt);
  const int ksteps = a.K / kKStep;
  uint32_t* err = a.err;

  if (tid == 0) {
    for (int s = 0; s < kStagesQ; ++s) {
      mbar_init(&sm.full_a[s], kNumDqWarps);
      mbar_init(&sm.full_b[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.tmem_full[i], 1);
      mbar_init(&sm.tmem_empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  // number of items this CTA owns
  uint32_t my_items = 0;
  if (blockIdx.x < n_items) my_items = (n_items - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const uint32_t total_steps = my_items * static_cast<uint32_t>(ksteps);

  if (warp == 4) {
    // ---------------- TMA producer: token tiles ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmap_b);
      uint32_t g = 0;
      bool ok = true;
      for (uint32_t i = 0; i < my_items && ok; ++i) {
        const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
        const uint32_t nbox = (w.rows + kBoxRows - 1) / kBoxRows;
        for (int ks = 0; ks < ksteps; ++ks, ++g) {
          const int s = static_cast<int>(g % kStagesQ);
          const uint32_t ph = (g / kStagesQ) & 1u;
          if (!mbar_wait(&sm.empty[s], ph ^ 1u, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&sm.full_b[s], nbox * kBoxRows * 128u);
          for (uint32_t b = 0; b < nbox; ++b)
            tma_load_2d(stage_b(s) + b * kBoxRows * 128, &tmap_b, &sm.full_b[s], ks * kKStep,
                        static_cast<int32_t>(w.row_start + b * kBoxRows));
        }
      }
      // drain: the last fill of every stage has landed
      const uint32_t issued = g;
      for (uint32_t q = (issued > kStagesQ ? issued - kStagesQ : 0); q < issued; ++q)
        mbar_wait(&sm.full_b[q % kStagesQ], (q / kStagesQ) & 1u, err);
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      for (uint32_t i = 0; i < my_items && ok; ++i) {
        const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
        const uint32_t n = (w.rows + 15u) & ~15u;
        const uint32_t idesc = umma_idesc_f16(128, n);
        const uint32_t acc = i & 1u;
        if (!mbar_wait(&sm.tmem_empty[acc], ((i >> 1) & 1u) ^ 1u, err)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem + acc * kTileN;
        for (int ks = 0; ks < ksteps; ++ks, ++g) {
          const int s = static_cast<int>(g % kStagesQ);
          const uint32_t ph = (g / kStagesQ) & 1u;
          if (!mbar_wait(&sm.full_a[s], ph, err) || !mbar_wait(&sm.full_b[s], ph, err)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint64_t da = umma_desc_sw128(smem_u32(stage_a(s)));
          const uint64_t db = umma_desc_sw128(smem_u32(stage_b(s)));
#pragma unroll
          for (int kk = 0; kk < kKStep / 16; ++kk)
            umma_f16_ss(d_tmem, da + 2u * kk, db + 2u * kk, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.empty[s]);
        }
        if (ok) umma_commit(&sm.tmem_full[acc]);
      }
    }
  } else if (warp >= kDqWarp0) {
    // ---------------- dequantisers ----------------
    const int d = tid - kDqWarp0 * 32;  // 0..255
    const int m = d & 127, h = d >> 7;
    uint4 pc[kPrefetch];
    __half ps[kPrefetch];
    // flattened (item, k-step) index -> loads
    auto fetch = [&](uint32_t step, int slot) {
      if (step >= total_steps) return;
      const uint32_t i = step / ksteps;
      const int ks = static_cast<int>(step % ksteps);
      const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
      const uint4* cp;
      const __half* sp;
      dq_source<MODE>(a, w, m, h, ks, &cp, &sp);
      pc[slot] = __ldg(cp);
      ps[slot] = __ldg(sp);
    };
#pragma unroll
    for (int q = 0; q < kPrefetch; ++q) fetch(q, q);
    bool ok = true;
    for (uint32_t g = 0; g < total_steps; ++g) {
      const int slot = static_cast<int>(g % kPrefetch);
      const uint4 c = pc[slot];
      const __half sc = ps[slot];
      fetch(g + kPrefetch, slot);
      const int s = static_cast<int>(g % kStagesQ);
      const uint32_t ph = (g / kStagesQ) & 1u;
      if (!mbar_wait(&sm.empty[s], ph ^ 1u, err)) { ok = false; break; }
      const __half2 s2 = __halves2half2(sc, sc);
      uint8_t* arow = stage_a(s) + m * 128;
      const uint32_t words[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        uint32_t o[4];
        nibbles_to_f16x2_scaled(words[wi], s2, o);
        const uint32_t chunk = static_cast<uint32_t>(h * 4 + wi) ^ static_cast<uint32_t>(m & 7);
        *reinterpret_cast<uint4*>(arow + chunk * 16) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.full_a[s]);
    }
    (void)ok;
  } else {
    // ---------------- epilogue: warps 0-3, TMEM lane quarter = warp ----------------
    const int q = warp;  // lanes 32q .. 32q+31
    for (uint32_t i = 0; i < my_items; ++i) {
      const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
      const uint32_t acc = i & 1u;
      if (!mbar_wait(&sm.tmem_full[acc], (i >> 1) & 1u, err)) break;
      tc_fence_after_sync();
      const uint32_t n = (w.rows + 15u) & ~15u;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(32 * q) << 16) + acc * kTileN;
      for (uint32_t c0 = 0; c0 < n; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tbase + c0, r);
        tmem_ld_wait();
        if (MODE == 0) {
          // rows 0-63 gate, 64-127 up: warps 2,3 hand their values over
          if (q >= 2) {
#pragma unroll
            for (int j = 0; j < 16; ++j) sm.xchg[((q - 2) * 32 + lane) * 17 + j] = __uint_as_float(r[j]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (q < 2) {
            const uint32_t f = w.wt * 64u + static_cast<uint32_t>(q * 32 + lane);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t col = c0 + j;
              if (col < w.rows) {
                const float g = __uint_as_float(r[j]);
                const float u = sm.xchg[(q * 32 + lane) * 17 + j];
                a.out[static_cast<size_t>(w.row_start + col) * a.out_cols + f] =
                    __float2half_rn(gate_act(a.act, g) * u);
              }
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        } else {
          const uint32_t dcol = w.wt * 128u + static_cast<uint32_t>(q * 32 + lane);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t col = c0 + j;
            if (col < w.rows)
              a.out[static_cast<size_t>(w.row_start + col) * a.out_cols + dcol] =
                  __float2half_rn(__uint_as_float(r[j]));
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tmem_empty[acc]);
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

size_t qmm_smem_bytes() { return static_cast<size_t>(kStagesQ) * (kABytes + kBBytes) + 1024; }

template <int MODE>
cudaError_t launch_qmm(const QmmParams& p, const CUtensorMap& tmap, cudaStream_t s) {
  QArgs a;
  a.ebase = p.experts.base;
  a.estride = p.experts.stride;
  a.off = p.experts.off;
  a.shared = p.experts.shared;
  a.soff = p.experts.shared_off;
  a.tiles = p.row_tiles;
  a.n_tiles = p.n_row_tiles;
  a.K = MODE == 0 ? p.D : p.F;
  a.n_wt = MODE == 0 ? p.F / 64 : p.D / 128;
  a.E = p.E;
  a.act = p.act;
  a.out_cols = MODE == 0 ? p.F : p.D;
  a.out = MODE == 0 ? p.act_buf : p.partials;
  a.err = p.err;
  const size_t smem = qmm_smem_bytes();
  cudaError_t e = allow_max_smem(qmm_kernel<MODE>);
  if (e != cudaSuccess) return e;
  qmm_kernel<MODE><<<p.num_sms, kThreadsQ, smem, s>>>(tmap, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qmm_gate_up(const QmmParams& p, cudaStream_t s) {
  if (p.D % 128 || p.F % 64) return cudaErrorInvalidValue;
  return launch_qmm<0>(p, p.maps[0], s);
}

cudaError_t launch_qmm_down(const QmmParams& p, cudaStream_t s) {
  if (p.D % 128 || p.F % 64) return cudaErrorInvalidValue;
  return launch_qmm<1>(p, p.maps[1], s);
}

int qmm_tile_rows() { return kTileN; }

}  // namespace tsg
