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
// B200 design (one persistent CTA per SM, warp-specialised, 27 warps):
//   * the tensor-core M operand is 128 weight rows (mode 0: 64 gate rows and
//     the 64 matching up rows, so one accumulator tile holds both halves of
//     act; mode 1: 128 down rows); the N operand is the row tile of sorted
//     token rows (<= 192, any multiple of 16), so a lightly routed expert
//     costs only the rows it has, and a full tile amortises the issue cost
//     of each MMA (~100-150 cycles per instruction on one thread) over
//     N = 192 columns;
//   * the dequantised weight tile lives in TENSOR MEMORY, not shared memory:
//     tcgen05.mma reads A from TMEM and only the token tile from shared
//     memory, which halves the shared-memory traffic per k-step;
//   * warp 5 streams the int4 code planes with TMA (3-D maps over
//     [expert][row][code byte], 128-byte boxes = four k-steps, 128-byte
//     swizzle so the dequantisers' 16-byte reads are bank-conflict free);
//     mode 0 brings the fp16 scales of the same four k-steps with two more
//     small boxes, mode 1 (whose scale rows are not 16-byte multiples) one
//     1-D bulk copy of the work item's scales;
//   * warps 7-22 (four per TMEM lane quarter: half h of a k-step, even or
//     odd k-steps) turn the codes into fp16 and store them into a TMEM ring
//     of A stages with tcgen05.st; alternating k-steps gives each warp two
//     k-steps of MMA time to cover the store's completion wait;
//   * warp 4 moves token tiles with TMA (one 192- or 128-row box for a
//     large tile, 16-row boxes for a small one; no multicast) into a
//     three-stage ring;
//   * warp 6 allocates TMEM (two 192-column fp32 accumulators + a two-stage
//     A ring of 64 columns each)
//     and issues tcgen05.mma (M=128, N=rows, K=16), committing to mbarriers;
//   * warps 0-3 and 23-26 (two per TMEM lane quarter, alternate 16-column
//     chunks) drain the accumulator with tcgen05.ld, apply the activation
//     or convert, and store fp16 rows.
// Every wait is bounded (tsg_common.cuh) and every wait that guards a
// warp-collective tcgen05 instruction is made warp-uniform, so a fault in
// the pipeline ends the kernel with an error flag instead of hanging.
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kTileN = 192;           // max token rows per tile (MMA N)
constexpr int kBoxRows = 16;          // small-tile TMA box height (rows)
constexpr int kKStep = 64;            // K per A/B stage (one 128-byte swizzle row)
constexpr int kBBytes = kTileN * 128;  // token rows x 64 fp16, 128-byte swizzle
constexpr int kCodeK = 4;              // k-steps per code stage (128 code bytes a row)
constexpr int kCodeBytes = 128 * 128;  // 128 weight rows x four k-steps of codes
constexpr int kScaleBoxBytes = 64 * 16;  // mode 0: 64 rows x 8 fp16 scales
constexpr int kStageK = 2;             // k-steps per A/B stage (one wait + one commit)
constexpr int kBStageBytes = kStageK * kBBytes;
constexpr int kAStages = 2;            // A ring in TMEM (2 x 64 columns after the accumulators)
constexpr int kMaxBStages = 3;         // B ring in shared memory
constexpr int kMaxCodeStages = 8;
constexpr int kThreadsQ = 27 * 32;
constexpr int kEpiWarp1 = 23;          // warps 0-3 and 23-26 drain the accumulators
constexpr int kEpiWarps = 8;
constexpr int kCodeWarp = 5;
constexpr int kMmaWarp = 6;   // shares its SMSP with epilogue warp 2, which only hands values over
constexpr int kDqWarp0 = 7;
constexpr int kNumDqWarps = 16;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCols = 2 * kTileN;  // columns [0, 384): two accumulators
constexpr uint32_t kAKStepCols = kKStep / 2;  // 64 fp16 of K per lane = 32 columns
constexpr uint32_t kAStageCols = kStageK * kAKStepCols;

struct QMaps {
  CUtensorMap b16, b128, b192;  // token rows: 16-, 128- and 192-row boxes
  CUtensorMap w0, w1;     // routed experts' code planes (mode 0: gate, up; 1: down)
  CUtensorMap ws0, ws1;   // the shared expert's
  CUtensorMap sc0, sc1;   // mode 0: routed gate / up scale planes
  CUtensorMap ssc0, ssc1; // mode 0: the shared expert's
};

template <int MODE>
struct CodeStage {
  // mode 0: gate codes, up codes, gate scales, up scales; mode 1: down codes
  static constexpr int bytes = MODE == 0 ? kCodeBytes + 2 * kScaleBoxBytes : kCodeBytes;
};

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
  int box128, box192;  // the 128- / 192-row token boxes are usable (enough rows)
  int b_stages;  // B ring depth
  int code_stages;
  uint32_t sc_bytes;  // one scale buffer, 128-byte aligned
  uint32_t c_off, s_off;  // code ring / scale buffers, from the aligned smem base
  __half* out;
  const unsigned long long* tile_out;  // mode 1, optional: per row tile, its rows' destination
  uint32_t* err;
};

struct SmemQ {
  uint64_t full_a[kAStages];   // A stored by the 16 dequantising warps
  uint64_t empty_a[kAStages];  // the MMAs that read it are done
  uint64_t full_b[kMaxBStages];
  uint64_t empty_b[kMaxBStages];
  uint64_t full_c[kMaxCodeStages];
  uint64_t empty_c[kMaxCodeStages];
  uint64_t full_s[2];
  uint64_t empty_s[2];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
};

struct WorkItem {
  uint32_t expert, row_start, rows, wt, tile;
  bool valid;
};

TSG_DEV WorkItem work_item(const QArgs& a, uint32_t n_items, uint32_t idx) {
  WorkItem w;
  w.valid = idx < n_items;
  if (!w.valid) return w;
  const uint32_t rt = idx / static_cast<uint32_t>(a.n_wt);
  w.wt = idx % static_cast<uint32_t>(a.n_wt);
  w.tile = rt;
  const RowTile t = a.tiles[rt];
  w.expert = t.expert;
  w.row_start = t.row_start;
  w.rows = t.rows;
  return w;
}

// Position in a ring of `n` stages: stage index and the parity of its fill.
struct Ring {
  int s = 0;
  uint32_t ph = 0;
  TSG_DEV void next(int n) {
    if (++s == n) { s = 0; ph ^= 1u; }
  }
};

// A bounded mbarrier wait whose outcome every lane of the warp shares, for
// waits that guard .sync.aligned instructions.
TSG_DEV bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  return __all_sync(0xffffffffu, mbar_sleep(bar, parity, err)) != 0;
}

template <int MODE, int ACT>
__global__ void __launch_bounds__(kThreadsQ, 1)
    qmm_kernel(const __grid_constant__ QMaps maps, const QArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ SmemQ sm;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - smem_u32(smem_raw));
  const int SB = a.b_stages, C = a.code_stages;
  constexpr int kCS = CodeStage<MODE>::bytes;
  auto stage_b = [&](int s) { return gbase + s * kBStageBytes; };
  auto stage_c = [&](int c) { return gbase + a.c_off + c * kCS; };
  auto scale_buf = [&](uint32_t b) { return gbase + a.s_off + b * a.sc_bytes; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t n_items = __ldg(a.n_tiles) * static_cast<uint32_t>(a.n_wt);
  const int ksteps = a.K / kKStep;
  const int stages_per_item = (ksteps + kStageK - 1) / kStageK;
  const uint32_t scale_row = static_cast<uint32_t>(a.K) / 16u;  // fp16 scale bytes per row
  uint32_t* err = a.err;

  if (tid == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&sm.full_a[s], kNumDqWarps);
      mbar_init(&sm.empty_a[s], 1);
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(&sm.full_b[s], 1);
      mbar_init(&sm.empty_b[s], 1);
    }
    for (int c = 0; c < C; ++c) {
      mbar_init(&sm.full_c[c], 1);
      mbar_init(&sm.empty_c[c], kNumDqWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.full_s[i], 1);
      mbar_init(&sm.empty_s[i], kNumDqWarps);
      mbar_init(&sm.tmem_full[i], 1);
      mbar_init(&sm.tmem_empty[i], kEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
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

  if (warp == 4) {
    // ---------------- TMA producer: token tiles ----------------
    if (lane == 0) {
      prefetch_tensormap(&maps.b16);
      if (a.box128) prefetch_tensormap(&maps.b128);
      if (a.box192) prefetch_tensormap(&maps.b192);
      uint32_t g = 0;
      Ring r;
      bool ok = true;
      for (uint32_t i = 0; i < my_items && ok; ++i) {
        const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
        // one box for the tile when a box that covers it exists (192 rows
        // for a tile of 129-192, 128 rows for 65-128; a box map exists only
        // when the buffer has that many rows), else 16-row boxes
        const uint32_t nbox = (w.rows + kBoxRows - 1) / kBoxRows;
        const CUtensorMap* bigmap = nullptr;
        uint32_t step_bytes = nbox * kBoxRows * 128u;
        if (w.rows > 128u) {
          if (a.box192) { bigmap = &maps.b192; step_bytes = 192u * 128u; }
        } else if (w.rows > 64u) {
          if (a.box128) { bigmap = &maps.b128; step_bytes = 128u * 128u; }
        }
        for (int j = 0; j < stages_per_item; ++j, ++g, r.next(SB)) {
          const int s = r.s;
          if (!mbar_sleep(&sm.empty_b[s], r.ph ^ 1u, err)) { ok = false; break; }
          const int kn = ksteps - kStageK * j < kStageK ? ksteps - kStageK * j : kStageK;
          mbar_arrive_expect_tx(&sm.full_b[s], static_cast<uint32_t>(kn) * step_bytes);
          for (int t = 0; t < kn; ++t) {
            const int ks = kStageK * j + t;
            uint8_t* dst = stage_b(s) + t * kBBytes;
            if (bigmap) {
              tma_load_2d(dst, bigmap, &sm.full_b[s], ks * kKStep, static_cast<int32_t>(w.row_start));
            } else {
              for (uint32_t b = 0; b < nbox; ++b)
                tma_load_2d(dst + b * kBoxRows * 128, &maps.b16, &sm.full_b[s], ks * kKStep,
                            static_cast<int32_t>(w.row_start + b * kBoxRows));
            }
          }
        }
      }
      // drain: the last fill of every stage has landed
      for (uint32_t q = (g > static_cast<uint32_t>(SB) ? g - SB : 0); q < g; ++q)
        mbar_sleep(&sm.full_b[q % SB], (q / SB) & 1u, err);
    }
  } else if (warp == kCodeWarp) {
    // ---------------- TMA producer: code planes and scales ----------------
    if (lane == 0) {
      prefetch_tensormap(&maps.w0);
      if (MODE == 0) {
        prefetch_tensormap(&maps.w1);
        prefetch_tensormap(&maps.sc0);
        prefetch_tensormap(&maps.sc1);
      }
      uint32_t cg = 0, scales_issued = 0;
      Ring r;
      bool ok = true;
      for (uint32_t i = 0; i < my_items && ok; ++i) {
        const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
        const bool sh = w.expert >= static_cast<uint32_t>(a.E);
        if (MODE == 1) {
          const uint8_t* blob =
              sh ? a.shared : a.ebase + static_cast<uint64_t>(w.expert) * a.estride;
          const ExpertOffsets& o = sh ? a.soff : a.off;
          const uint32_t b = i & 1u;
          if (!mbar_sleep(&sm.empty_s[b], ((i >> 1) & 1u) ^ 1u, err)) break;
          const uint32_t all = 128u * scale_row;
          mbar_arrive_expect_tx(&sm.full_s[b], all);
          bulk_load(scale_buf(b), blob + o.down_s + static_cast<size_t>(w.wt) * all, all,
                    &sm.full_s[b]);
          ++scales_issued;
        }
        const CUtensorMap* m0 = sh ? &maps.ws0 : &maps.w0;
        const CUtensorMap* m1 = sh ? &maps.ws1 : &maps.w1;
        const CUtensorMap* q0 = sh ? &maps.ssc0 : &maps.sc0;
        const CUtensorMap* q1 = sh ? &maps.ssc1 : &maps.sc1;
        const int32_t z = sh ? 0 : static_cast<int32_t>(w.expert);
        const int32_t y = static_cast<int32_t>(w.wt * (MODE == 0 ? 64u : 128u));
        for (int k0 = 0; k0 < ksteps; k0 += kCodeK, ++cg, r.next(C)) {
          const int cs = r.s;
          if (!mbar_sleep(&sm.empty_c[cs], r.ph ^ 1u, err)) { ok = false; break; }
          uint8_t* dst = stage_c(cs);
          mbar_arrive_expect_tx(&sm.full_c[cs], kCS);
          // x counts code bytes (32 per k-step) in the code planes and fp16
          // scale groups (2 per k-step) in the scale planes
          tma_load_3d(dst, m0, &sm.full_c[cs], k0 * 32, y, z);
          if (MODE == 0) {
            tma_load_3d(dst + kCodeBytes / 2, m1, &sm.full_c[cs], k0 * 32, y, z);
            tma_load_3d(dst + kCodeBytes, q0, &sm.full_c[cs], k0 * 2, y, z);
            tma_load_3d(dst + kCodeBytes + kScaleBoxBytes, q1, &sm.full_c[cs], k0 * 2, y, z);
          }
        }
      }
      // drain: the last fill of every code stage and scale buffer has landed
      for (uint32_t q = (cg > static_cast<uint32_t>(C) ? cg - C : 0); q < cg; ++q)
        mbar_sleep(&sm.full_c[q % C], (q / C) & 1u, err);
      for (uint32_t q = (scales_issued > 2 ? scales_issued - 2 : 0); q < scales_issued; ++q)
        mbar_sleep(&sm.full_s[q & 1u], (q >> 1) & 1u, err);
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      Ring ra, rb;  // A ring (TMEM), B ring (shared memory)
      bool ok = true;
      for (uint32_t i = 0; i < my_items && ok; ++i) {
        const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
        const uint32_t n = (w.rows + 15u) & ~15u;
        const uint32_t idesc = umma_idesc_f16(128, n);
        const uint32_t acc = i & 1u;
        if (!mbar_sleep(&sm.tmem_empty[acc], ((i >> 1) & 1u) ^ 1u, err)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem + acc * kTileN;
        bool ready = false;  // the next stage's A and B were seen ready already
        for (int j = 0; j < stages_per_item; ++j, ra.next(kAStages), rb.next(SB)) {
          if (!ready &&
              (!mbar_sleep(&sm.full_a[ra.s], ra.ph, err) || !mbar_sleep(&sm.full_b[rb.s], rb.ph, err))) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a_tmem = tmem + kAccCols + static_cast<uint32_t>(ra.s) * kAStageCols;
          const uint32_t b0 = smem_u32(stage_b(rb.s));
          umma_f16_ts_k64(d_tmem, a_tmem, umma_desc_sw128(b0), idesc, j > 0 ? 1u : 0u);
          if (kStageK * j + 1 < ksteps)
            umma_f16_ts_k64(d_tmem, a_tmem + kAKStepCols, umma_desc_sw128(b0 + kBBytes), idesc, 1u);
          // look at the next stage's barriers before the commits, so that
          // the answer is back by the time the loop needs it
          Ring na = ra, nb = rb;
          na.next(kAStages);
          nb.next(SB);
          ready = j + 1 < stages_per_item && mbar_test_wait(&sm.full_a[na.s], na.ph) &&
                  mbar_test_wait(&sm.full_b[nb.s], nb.ph);
          umma_commit(&sm.empty_a[ra.s]);
          umma_commit(&sm.empty_b[rb.s]);
        }
        if (ok) umma_commit(&sm.tmem_full[acc]);
      }
    }
  } else if (warp >= kDqWarp0 && warp < kDqWarp0 + kNumDqWarps) {
    // ---------------- dequantisers: codes -> fp16 A tile in TMEM ----------------
    // Warp w serves TMEM lanes 32*(w%4).. (its hardware lane quarter); role
    // r = (w - 7) / 4 picks half h = r & 1 of a k-step and which k-step
    // (par = r >> 1) of each two-k-step A stage it fills.  Thread = one
    // weight row.  All 16 warps arrive on every stage's `full` barrier, a
    // warp whose k-step lies past the end of the item without storing.
    const int r = (warp - kDqWarp0) >> 2;
    const int q = warp & 3, h = r & 1;
    const int par = r >> 1;
    // Mode 0 interleaves gate and up rows across the TMEM lanes so that each
    // epilogue warp holds both halves of its act values: lanes 32q + [0,16)
    // are gate rows f0 + 16q + [0,16), lanes 32q + [16,32) the matching up
    // rows.  `m` is the row inside the code stage (gate rows 0-63, up 64-127).
    const int m = MODE == 0 ? ((lane & 16) << 2) + 16 * q + (lane & 15) : 32 * q + lane;
    const uint32_t xr = static_cast<uint32_t>(m & 7);  // 128-byte swizzle of row m
    const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * q) << 16) + kAccCols +
                           static_cast<uint32_t>(par) * kAKStepCols + static_cast<uint32_t>(h) * 16u;
    Ring ra, rc;  // A/B ring position, code ring position
    int pend = -1;  // A stage whose stores still have to be published
    bool ok = true;
    for (uint32_t i = 0; i < my_items && ok; ++i) {
      const uint32_t b = i & 1u;
      const uint8_t* srow = nullptr;
      if (MODE == 1) {
        if (!warp_wait(&sm.full_s[b], (i >> 1) & 1u, err)) { ok = false; break; }
        srow = scale_buf(b) + m * scale_row + 2 * h;
      }
      for (int k0 = 0; k0 < ksteps; k0 += kCodeK) {
        const int cs = rc.s;
        if (!warp_wait(&sm.full_c[cs], rc.ph, err)) { ok = false; break; }
        const uint8_t* cst = stage_c(cs);
        uint4 sc8 = make_uint4(0u, 0u, 0u, 0u);  // mode 0: row m's 8 scales of the stage
        if (MODE == 0) sc8 = *reinterpret_cast<const uint4*>(cst + kCodeBytes + m * 16);
#pragma unroll
        for (int jj = 0; jj < kCodeK / kStageK; ++jj) {
          const int kbase = k0 + kStageK * jj;  // first k-step of this A stage
          if (kbase >= ksteps) break;
          const int s = ra.s;
          const uint32_t ph = ra.ph;
          ra.next(kAStages);
          const int j = kStageK * jj + par;      // my k-step inside the code stage
          const bool have = k0 + j < ksteps;
          uint32_t o[16];
          if (have) {
            const uint32_t chunk = static_cast<uint32_t>(2 * j + h) ^ xr;
            const uint4 c = *reinterpret_cast<const uint4*>(cst + m * 128 + chunk * 16);
            __half sc;
            if (MODE == 0) {
              const uint32_t wv = j == 0 ? sc8.x : j == 1 ? sc8.y : j == 2 ? sc8.z : sc8.w;
              const unsigned short bits =
                  static_cast<unsigned short>(h ? (wv >> 16) : (wv & 0xFFFFu));
              sc = __ushort_as_half(bits);
            } else {
              sc = *reinterpret_cast<const __half*>(srow + 4 * (k0 + j));
            }
            const __half2 s2 = __halves2half2(sc, sc);
            uint32_t t[4];
            nibbles_to_f16x2_scaled(c.x, s2, t);
            o[0] = t[0]; o[1] = t[1]; o[2] = t[2]; o[3] = t[3];
            nibbles_to_f16x2_scaled(c.y, s2, t);
            o[4] = t[0]; o[5] = t[1]; o[6] = t[2]; o[7] = t[3];
            nibbles_to_f16x2_scaled(c.z, s2, t);
            o[8] = t[0]; o[9] = t[1]; o[10] = t[2]; o[11] = t[3];
            nibbles_to_f16x2_scaled(c.w, s2, t);
            o[12] = t[0]; o[13] = t[1]; o[14] = t[2]; o[15] = t[3];
          }
          if (pend >= 0) {  // publish the previous stage while this one was converted
            tmem_st_wait();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.full_a[pend]);
            pend = -1;
          }
          if (!warp_wait(&sm.empty_a[s], ph ^ 1u, err)) { ok = false; break; }
          tc_fence_after_sync();
          if (have) tmem_st16(t_row + static_cast<uint32_t>(s) * kAStageCols, o);
          pend = s;
        }
        if (!ok) break;
        // this code stage is used up (its values are in registers or TMEM)
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty_c[cs]);
        rc.next(C);
      }
      if (!ok) break;
      if (MODE == 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty_s[b]);
      }
    }
    if (pend >= 0) {
      tmem_st_wait();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.full_a[pend]);
    }
  } else if (warp < 4 || warp >= kEpiWarp1) {
    // ---------------- epilogue: warps 0-3 and 23-26 ----------------
    // Two warps per TMEM lane quarter (q = warp % 4), taking alternate
    // 16-column chunks.  A failed wait does not leave the loop: the warp
    // only skips the TMEM reads and the stores.
    const int q = warp & 3;  // lanes 32q .. 32q+31
    const uint32_t c_first = warp < 4 ? 0u : 16u;
    const bool upper = lane >= 16;
    for (uint32_t i = 0; i < my_items; ++i) {
      const WorkItem w = work_item(a, n_items, blockIdx.x + i * gridDim.x);
      const uint32_t acc = i & 1u;
      const bool ok = warp_wait(&sm.tmem_full[acc], (i >> 1) & 1u, err);
      tc_fence_after_sync();
      const uint32_t n = (w.rows + 15u) & ~15u;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(32 * q) << 16) + acc * kTileN;
      for (uint32_t c0 = c_first; ok && c0 < n; c0 += 32) {
        uint32_t r[16];
        tmem_ld16(tbase + c0, r);
        tmem_ld_wait();
        if (MODE == 0) {
          // lane l < 16 holds gate(f, c0 + j), lane l + 16 up(f, c0 + j).  The
          // low half-warp finishes columns c0..c0+7, the high half c0+8..c0+15:
          // each sends the other the 8 values it lacks.
          const uint32_t f = w.wt * 64u + static_cast<uint32_t>(16 * q + (lane & 15));
          const uint32_t cb = c0 + (upper ? 8u : 0u);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float mine = __uint_as_float(upper ? r[j + 8] : r[j]);
            const float give = __uint_as_float(upper ? r[j] : r[j + 8]);
            const float other = __shfl_xor_sync(0xffffffffu, give, 16);
            const float gv = upper ? other : mine;
            const float uv = upper ? mine : other;
            const uint32_t col = cb + j;
            if (col < w.rows)
              a.out[static_cast<size_t>(w.row_start + col) * a.out_cols + f] =
                  __float2half_rn(gate_act_fast(ACT, gv) * uv);
          }
        } else {
          const uint32_t dcol = w.wt * 128u + static_cast<uint32_t>(q * 32 + lane);
          __half* ob = a.tile_out ? reinterpret_cast<__half*>(a.tile_out[w.tile])
                                  : a.out + static_cast<size_t>(w.row_start) * a.out_cols;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t col = c0 + j;
            if (col < w.rows)
              ob[static_cast<size_t>(col) * a.out_cols + dcol] = __float2half_rn(__uint_as_float(r[j]));
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tmem_empty[acc]);
    }
    // rows written into another rank's memory are visible there before the
    // collective that follows this kernel
    if (MODE == 1 && a.tile_out) __threadfence_system();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Token rows of a [rows][cols] fp16 matrix, 64-element (128-byte) wide boxes
// of `box_rows` rows in the 128-byte swizzle the UMMA descriptor reads.
bool encode_rows(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                 uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Int4 code planes of `n` experts, [n][rows][row_bytes] bytes with experts
// `nstride` bytes apart: boxes of 128 bytes (four k-steps) x `box_rows`
// rows, 128-byte swizzle.
bool encode_codes(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
                  uint64_t n, uint64_t nstride, uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {row_bytes, rows, n};
  const cuuint64_t strides[2] = {row_bytes, nstride};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp16 scale planes of `n` experts, [n][rows][groups]: boxes of 8 groups
// (four k-steps, 16 bytes) x 64 rows, no swizzle.  Needs groups * 2 to be a
// multiple of 16 bytes.
bool encode_scales(CUtensorMap* map, const void* base, uint64_t groups, uint64_t rows,
                   uint64_t n, uint64_t nstride) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {groups, rows, n};
  const cuuint64_t strides[2] = {groups * 2, nstride};
  const cuuint32_t box[3] = {8, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE>
cudaError_t launch_qmm(const QmmParams& p, cudaStream_t s) {
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
  a.tile_out = MODE == 1 ? p.tile_out : nullptr;
  a.err = p.err;

  // token rows
  const uint64_t rows = p.n_rows_total > 0 ? static_cast<uint64_t>(p.n_rows_total) : 1u;
  const __half* bsrc = MODE == 0 ? p.xp : p.act_buf;
  QMaps maps;
  if (!encode_rows(&maps.b16, bsrc, rows, static_cast<uint64_t>(a.K), kBoxRows))
    return cudaErrorInvalidValue;
  a.box128 = rows >= 128u ? 1 : 0;
  a.box192 = rows >= 192u ? 1 : 0;
  maps.b128 = maps.b16;
  maps.b192 = maps.b16;
  if (a.box128 && !encode_rows(&maps.b128, bsrc, rows, static_cast<uint64_t>(a.K), 128u))
    return cudaErrorInvalidValue;
  if (a.box192 && !encode_rows(&maps.b192, bsrc, rows, static_cast<uint64_t>(a.K), 192u))
    return cudaErrorInvalidValue;
  // code planes (and, for mode 0, scale planes) of the routed and shared experts
  const uint64_t row_bytes = static_cast<uint64_t>(a.K) / 2;
  const uint64_t groups = static_cast<uint64_t>(a.K) / 32;
  const uint64_t n_rows = MODE == 0 ? static_cast<uint64_t>(p.F) : static_cast<uint64_t>(p.D);
  const uint32_t box_rows = MODE == 0 ? 64u : 128u;
  const uint64_t n_exp = p.E > 0 ? static_cast<uint64_t>(p.E) : 1u;
  const uint64_t est = p.experts.stride ? p.experts.stride : row_bytes * n_rows;
  const ExpertOffsets& o = p.experts.off;
  const ExpertOffsets& so = p.experts.shared_off;
  const uint32_t o0 = MODE == 0 ? o.gate_w : o.down_w;
  const uint32_t o1 = MODE == 0 ? o.up_w : o.down_w;
  if (!encode_codes(&maps.w0, p.experts.base + o0, row_bytes, n_rows, n_exp, est, box_rows) ||
      !encode_codes(&maps.w1, p.experts.base + o1, row_bytes, n_rows, n_exp, est, box_rows))
    return cudaErrorInvalidValue;
  maps.ws0 = maps.w0;
  maps.ws1 = maps.w1;
  if (p.experts.shared) {
    const uint32_t s0 = MODE == 0 ? so.gate_w : so.down_w;
    const uint32_t s1 = MODE == 0 ? so.up_w : so.down_w;
    const uint64_t one = row_bytes * n_rows;
    if (!encode_codes(&maps.ws0, p.experts.shared + s0, row_bytes, n_rows, 1, one, box_rows) ||
        !encode_codes(&maps.ws1, p.experts.shared + s1, row_bytes, n_rows, 1, one, box_rows))
      return cudaErrorInvalidValue;
  }
  maps.sc0 = maps.sc1 = maps.ssc0 = maps.ssc1 = maps.w0;  // unused in mode 1
  if (MODE == 0) {
    if ((groups * 2) % 16) return cudaErrorInvalidValue;  // D % 256 == 0 guarantees it
    if (!encode_scales(&maps.sc0, p.experts.base + o.gate_s, groups, n_rows, n_exp, est) ||
        !encode_scales(&maps.sc1, p.experts.base + o.up_s, groups, n_rows, n_exp, est))
      return cudaErrorInvalidValue;
    maps.ssc0 = maps.sc0;
    maps.ssc1 = maps.sc1;
    if (p.experts.shared) {
      const uint64_t one = groups * 2 * n_rows;
      if (!encode_scales(&maps.ssc0, p.experts.shared + so.gate_s, groups, n_rows, 1, one) ||
          !encode_scales(&maps.ssc1, p.experts.shared + so.up_s, groups, n_rows, 1, one))
        return cudaErrorInvalidValue;
    }
  }

  // shared-memory plan: A/B ring, code ring, (mode 1) two scale buffers
  void (*kern)(QMaps, QArgs) =
      (MODE == 0 && p.act == 1) ? qmm_kernel<MODE, 1> : qmm_kernel<MODE, 0>;
  cudaError_t e = allow_max_smem(kern);
  if (e != cudaSuccess) return e;
  int dev = 0, optin = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa;
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return e;
  a.sc_bytes = MODE == 1 ? (128u * static_cast<uint32_t>(a.K) / 16u + 127u) & ~127u : 0u;
  int S = kMaxBStages, C = kMaxCodeStages;
  auto need = [&]() {
    return static_cast<size_t>(1024) + static_cast<size_t>(S) * kBStageBytes +
           static_cast<size_t>(C) * CodeStage<MODE>::bytes + 2u * static_cast<size_t>(a.sc_bytes);
  };
  while (need() + fa.sharedSizeBytes > static_cast<size_t>(optin)) {
    if (C > 3) --C;
    else if (S > 2) --S;
    else return cudaErrorInvalidValue;
  }
  a.b_stages = S;
  a.code_stages = C;
  a.c_off = static_cast<uint32_t>(S * kBStageBytes);
  a.s_off = a.c_off + static_cast<uint32_t>(C * CodeStage<MODE>::bytes);
  kern<<<p.num_sms, kThreadsQ, need(), s>>>(maps, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qmm_gate_up(const QmmParams& p, cudaStream_t s) {
  if (p.D % 256 || p.F % 64) return cudaErrorInvalidValue;
  return launch_qmm<0>(p, s);
}

cudaError_t launch_qmm_down(const QmmParams& p, cudaStream_t s) {
  if (p.D % 128 || p.F % 64) return cudaErrorInvalidValue;
  return launch_qmm<1>(p, s);
}

int qmm_tile_rows() { return kTileN; }

}  // namespace tsg
