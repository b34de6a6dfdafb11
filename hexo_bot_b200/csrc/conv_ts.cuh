// HexNodeConv (7 taps; 19 for the ray-tap conv) for short positions, with the
// A operand built on chip.
//
//   out[m, :] = epilogue( sum_t X[src(m, t), :] @ W_t )      (model.py:346-370)
//
// Tiles are aligned to positions: one tile = `ppt` whole positions
// (ppt * cells <= 128 output rows; 2 positions of 61 cells in the disk
// regime). The rows of those positions (the "window": ppt * rows-per-position
// rows of X, contiguous in memory) arrive in shared memory with one 2D TMA
// load per 64-column box, so every X row crosses from L2 once per tile instead
// of once per tap. Four A-builder warps (one per TMEM lane quadrant, one
// output row per thread) gather each 64-wide K chunk of their row's 7 taps
// from the window and store it into TMEM; the MMA warp runs tcgen05.mma with
// A from TMEM and the weight chunk (streamed through a TMA ring) from shared
// memory, so shared-memory bandwidth is spent on the weights and the gather
// reads only. The epilogue is the eight-warp epilogue of gemm_ws_kernel.
//
// Warp roles (480 threads; 608 in the light instantiation): 0-7 epilogue,
// 8 MMA issue, 9 weight producer, 10-13 A builders, 14 window producer,
// 15-18 the second A-builder set (light instantiation only).
#pragma once

#include "gemm.cuh"

namespace sb {

constexpr int kConvWarps = 15;
constexpr int kConvThreads = kConvWarps * 32;
// The light instantiation (no residual, no TMA epilogue) adds a second set of
// four A-builder warps (warps 15-18): its registers fit 19 warps without
// spilling, and the builders are on the per-stage critical path.
constexpr int kConvBuilder1 = 15;
__host__ __device__ constexpr int conv_ts_threads(bool heavy) { return heavy ? kConvThreads : kConvThreads + 128; }
constexpr int kConvMmaWarp = 8;
constexpr int kConvWProducer = 9;
constexpr int kConvBuilder0 = 10;
constexpr int kConvWinProducer = 14;
constexpr int kConvMaxStages = 8;
constexpr int kConvStageChunks = 2;  // 64-wide K chunks per ring stage (one barrier round trip per 8 MMAs)

struct ConvTsGeom {
  int ppt;        // positions per tile (1, 2 or 4)
  int cells;      // output rows per position (<= 128 / ppt)
  int xrows;      // X rows per position (window rows = ppt * xrows)
  int npos;       // positions
  int tokoff;     // output rows before the cells in each position's block (seq layout: 8 tokens)
};
// TMEM lane (tile row) r holds cell r % lpb of the tile's position r / lpb,
// lpb = 128 / ppt lanes per position: each 32-lane quadrant covers one
// contiguous run of one position's rows (lanes past `cells` are padding).

__host__ __device__ constexpr int conv_win_box_bytes(int win_rows) { return (win_rows * 128 + 1023) / 1024 * 1024; }
// tma_epi: the epilogue stages its chunks for TMA stores (residual convs).
__host__ __device__ constexpr int conv_ts_smem_bytes(int c, int stages, int win_rows, bool tma_epi = false) {
  return 1024 + stages * kConvStageChunks * c * 128 + 2 * (c / 64) * conv_win_box_bytes(win_rows) + kEpiSmemBytes +
         (tma_epi ? kEpiTmaBytes + 1024 : 0) + 8 * (2 * stages + 8 + 8) + 16;
}
// Ring depth: limited by shared memory and by TMEM (two C-column accumulators
// plus 32 columns per A chunk of each stage, within 512 columns).
__host__ __device__ constexpr int conv_ts_stages(int c, int win_rows, bool tma_epi = false) {
  int s = kConvMaxStages;
  while (s > 2 && (conv_ts_smem_bytes(c, s, win_rows, tma_epi) > 227 * 1024 ||
                   2 * ((c + 31) / 32 * 32) + 32 * kConvStageChunks * s > 512))
    --s;
  return s;
}

template <typename T, bool HEAVY, int TAPS = 7>
__global__ void __launch_bounds__(conv_ts_threads(HEAVY), 1)
    conv_ts_kernel(const GemmArgs a, const ConvTsGeom geo, const __grid_constant__ CUtensorMap tmap_x,
                   const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_o16,
                   const __grid_constant__ CUtensorMap tmap_o32, int stages) {
  if (a.skip_flag) {
    pdl_wait();
    if (*reinterpret_cast<const volatile int*>(a.skip_flag) == a.skip_value) return;
  }
  extern __shared__ uint8_t smem_raw[];
  constexpr int kSets = HEAVY ? 1 : 2;  // A-builder warp sets
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = stages;
  const int C = a.n_total;  // == a.bn == a.cin
  // Window: C / 64 boxes of 64 columns (128-byte swizzled rows) when the input
  // has C channels; one unswizzled box of cin columns for a narrow input (the
  // stem's 16 feature planes), whose K chunks then span several taps.
  const int cin = a.cin;
  const bool narrow = cin < 64;
  const int nbox = narrow ? 1 : C / 64;
  const int win_row_bytes = narrow ? cin * 2 : 128;  // bytes of one window row in one box
  const int win_rows = geo.ppt * geo.xrows;
  const int box_bytes = conv_win_box_bytes(win_rows);
  const int lpb = kBlockM / geo.ppt;  // TMEM lanes per position

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t chunk_bytes = C * 128;                 // one 64-wide K chunk of the weights
  const uint32_t stage_bytes = kConvStageChunks * chunk_bytes;
  const uint32_t win_off = S * stage_bytes;                             // [2][nbox][box_bytes]
  const uint32_t epi_off = win_off + 2 * (C / 64) * box_bytes;          // as sized by conv_ts_smem_bytes
  float* vecs = reinterpret_cast<float*>(gbase + epi_off);
  float4* xch_all = reinterpret_cast<float4*>(gbase + epi_off + kEpiVecFloats * 4);
  // TMA epilogue staging (heavy instantiation), 1024-aligned
  const uint32_t stg_off = (epi_off + kEpiSmemBytes + 1023u) & ~1023u;
  const uint32_t bar0 = base + (HEAVY ? stg_off + kEpiTmaBytes : epi_off + kEpiSmemBytes);
  // Stage s = weight chunk in shared memory + A chunk in TMEM slot s: full
  // when the TMA bytes landed and the four A builders stored their rows;
  // empty when the MMAs that read both completed.
  const uint32_t full_bar = bar0;                         // [S]
  const uint32_t empty_bar = full_bar + 8 * S;            // [S]
  const uint32_t winf_bar = empty_bar + 8 * S;            // [2]   window landed
  const uint32_t wine_bar = winf_bar + 16;                // [2]   window consumed
  const uint32_t accf_bar = wine_bar + 16;                // [2]
  const uint32_t acce_bar = accf_bar + 16;                // [2]
  const uint32_t rload_bar = acce_bar + 16;               // [8] residual loads (TMA epilogue)
  const uint32_t tmem_slot = rload_bar + 64;
  volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const int acc_cols = (C + 31) & ~31;
  const uint32_t a_col0 = 2 * acc_cols;  // A chunk buffers follow the two accumulators
  const uint32_t ncols = 512;

  const int tiles = (geo.npos + geo.ppt - 1) / geo.ppt;
  const int nk = a.kpad / kChunkK;  // 7 * C / 64 chunks per tile
  const int nst = (nk + kConvStageChunks - 1) / kConvStageChunks;  // ring stages per tile

  pdl_launch_dependents();
  if (warp == kConvMmaWarp) {
    tmem_alloc(tmem_slot, ncols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar + 8 * s, 1 + 4 * kSets);
      mbar_init(empty_bar + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(winf_bar + 8 * i, 1);
      mbar_init(wine_bar + 8 * i, 4 * kSets);
      mbar_init(accf_bar + 8 * i, 1);
      mbar_init(acce_bar + 8 * i, kEpiWarps);
    }
    for (int i = 0; i < kEpiWarps; ++i) mbar_init(rload_bar + 8 * i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;
  bool ok = true;
  // Roles that read activations or write global memory wait for the previous
  // kernel; the weight producer and the MMA issuer (shared memory and TMEM
  // only) start filling the weight ring during that wait.
  if (warp != kConvWProducer && warp != kConvMmaWarp) pdl_wait();

  if (warp == kConvWinProducer) {
    // ------------------------------------------------------------ window producer
    if (lane == 0) {
      int j = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
        const int wb = j & 1;
        if (ok && !mbar_wait_sleep(wine_bar + 8 * wb, ((j >> 1) & 1) ^ 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
        }
        if (!ok) break;
        mbar_arrive_expect_tx(winf_bar + 8 * wb, nbox * win_rows * win_row_bytes);
        const int row0 = t * geo.ppt * geo.xrows;
        for (int bx = 0; bx < nbox; ++bx)
          tma_load_2d(base + win_off + (wb * nbox + bx) * box_bytes, &tmap_x, bx * 64, row0, winf_bar + 8 * wb);
      }
    }
    __syncwarp();
  } else if (warp == kConvWProducer) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;  // ring slot and its phase, advanced per stage (no division)
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        for (int q = 0; q < nst; ++q) {
          const int nc = min(kConvStageChunks, nk - q * kConvStageChunks);
          if (ok && !mbar_wait_sleep(empty_bar + 8 * s, ph ^ 1)) {
            ok = false;
            if (a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
          }
          if (!ok) break;
          mbar_arrive_expect_tx(full_bar + 8 * s, nc * chunk_bytes);
          for (int h = 0; h < nc; ++h)
            tma_load_2d(base + s * stage_bytes + h * chunk_bytes, &tmap_w, (q * kConvStageChunks + h) * kChunkK, 0,
                        full_bar + 8 * s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if ((warp >= kConvBuilder0 && warp < kConvBuilder0 + 4) || warp >= kConvBuilder1) {
    // ------------------------------------------------------------ A builders
    // kSets sets of four warps (one per TMEM lane quadrant in each set); with
    // two sets, set bs builds chunk bs of every two-chunk stage
    const int bs = warp >= kConvBuilder1 ? 1 : 0;
    const int quad = warp & 3;        // TMEM lanes [32 quad, 32 quad + 32)
    const int row = quad * 32 + lane; // row within the tile
    const uint32_t tlane = tmem_base + ((uint32_t)(quad * 32) << 16);
    uint32_t ac = 0;                  // A chunks produced
    int bslot = 0;                    // ring slot of the next stage and its phase (advanced per stage)
    uint32_t bph = 0;
    int j = 0;
    // this thread's TAPS tap rows for tile t (window-local, -1 = zero)
    const int rp = row / lpb, ri = row - rp * lpb;  // position in the tile, cell in the position
    auto load_src = [&](int t, int (&src)[TAPS]) {
      const int pos = t * geo.ppt + rp;
      const int m = pos * geo.cells + ri;
      const bool live = ri < geo.cells && pos < geo.npos && m < a.M && t < tiles;
      const int w0 = t * geo.ppt * geo.xrows;
#pragma unroll
      for (int k = 0; k < TAPS; ++k) {
        int v = live ? __ldg(a.gidx + (long long)m * TAPS + k) : -1;
        v = v >= 0 ? v - w0 : -1;
        src[k] = (v >= 0 && v < win_rows) ? v : -1;
      }
    };
    // 7 taps: the next tile's rows are prefetched during this tile; 19 taps:
    // loaded at the tile start (two sets of 19 registers would spill)
    constexpr bool kPrefetch = TAPS <= 7;
    int src[TAPS], nxt[kPrefetch ? TAPS : 1];
    if constexpr (kPrefetch) load_src(blockIdx.x, nxt);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      if constexpr (kPrefetch) {
#pragma unroll
        for (int k = 0; k < TAPS; ++k) src[k] = nxt[k];
        load_src(t + gridDim.x, nxt);  // prefetch the next tile's rows
      } else {
        load_src(t, src);
      }
      const int wb = j & 1;
      const bool got = ok && mbar_wait_sleep(winf_bar + 8 * wb, (j >> 1) & 1);
      ok = __all_sync(0xffffffffu, got) != 0;
      if (!ok) {
        if (lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
        break;
      }
      const uint32_t win = base + win_off + wb * nbox * box_bytes;  // shared-window address
      // gather chunk c of this thread's row from the window (zeros for a
      // missing tap) into 32 registers
      auto gather = [&](int c, uint32_t (&v)[32]) {
        const int k0 = c * kChunkK;
        if (narrow) {
          // 8 pieces of 8 channels; piece p is channel (k0 + 8p) % cin of tap
          // (k0 + 8p) / cin (taps past the seventh are the K padding: zeros)
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int kk = k0 + 8 * p;
            const int tap = kk / cin;
            int r = src[0];
#pragma unroll
            for (int k = 1; k < TAPS; ++k) r = tap == k ? src[k] : r;
            r = tap < TAPS ? r : -1;
            const int rr = r < 0 ? 0 : r;
            const uint32_t keep = r < 0 ? 0u : 0xffffffffu;
            const uint4 u = lds128(win + rr * win_row_bytes + (kk - tap * cin) * 2);
            v[4 * p] = u.x & keep;
            v[4 * p + 1] = u.y & keep;
            v[4 * p + 2] = u.z & keep;
            v[4 * p + 3] = u.w & keep;
          }
          return;
        }
        const int tap = k0 / C;
        const int bx = (k0 - tap * C) >> 6;
        int r = src[0];
#pragma unroll
        for (int k = 1; k < TAPS; ++k) r = tap == k ? src[k] : r;  // registers, no local array
        // branch-free: a missing tap reads row 0 and is masked to zero
        const int rr = r < 0 ? 0 : r;
        const uint32_t keep = r < 0 ? 0u : 0xffffffffu;
        const uint32_t rowp = win + bx * box_bytes + rr * 128;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const uint4 u = lds128(rowp + ((p ^ (rr & 7)) << 4));
          v[4 * p] = u.x & keep;
          v[4 * p + 1] = u.y & keep;
          v[4 * p + 2] = u.z & keep;
          v[4 * p + 3] = u.w & keep;
        }
      };
      uint32_t va[32], vb[32];
      if constexpr (kSets == 1) {
        // Software pipeline: the gather of chunk c + 1 overlaps the TMEM store
        // of chunk c; a stage (two chunks) is published once its stores have
        // completed.
        gather(0, va);
        for (int q = 0; q < nst; ++q) {
          const int slot = bslot;
          const bool free_ok = mbar_wait(empty_bar + 8 * slot, bph ^ 1);
          if (++bslot == S) {
            bslot = 0;
            bph ^= 1;
          }
          ok = __all_sync(0xffffffffu, free_ok) != 0;
          if (!ok) {
            if (lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
            break;
          }
          tc_fence_after();
          const int c0 = q * kConvStageChunks;
          __syncwarp();
          tmem_st32(tlane + a_col0 + slot * (32 * kConvStageChunks), va);
          if (c0 + 1 < nk) gather(c0 + 1, vb);
          __syncwarp();
          if (c0 + 1 < nk) tmem_st32(tlane + a_col0 + slot * (32 * kConvStageChunks) + 32, vb);
          if (c0 + 2 < nk) gather(c0 + 2, va);
          __syncwarp();
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(full_bar + 8 * slot);
        }
      } else {
        // Two sets: set bs stores chunk bs of each stage; the gather of its
        // chunk of the next stage overlaps the store of the current one.
        auto step = [&](int q, uint32_t (&cur)[32], uint32_t (&nxt)[32]) -> bool {
          const int slot = bslot;
          const bool free_ok = mbar_wait(empty_bar + 8 * slot, bph ^ 1);
          if (++bslot == S) {
            bslot = 0;
            bph ^= 1;
          }
          if (!__all_sync(0xffffffffu, free_ok)) return false;
          tc_fence_after();
          const int c = q * kConvStageChunks + bs;
          __syncwarp();
          if (c < nk) tmem_st32(tlane + a_col0 + slot * (32 * kConvStageChunks) + bs * 32, cur);
          if (c + kConvStageChunks < nk) gather(c + kConvStageChunks, nxt);
          __syncwarp();
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(full_bar + 8 * slot);
          return true;
        };
        if (bs < nk) gather(bs, va);
        for (int q = 0; q < nst && ok; q += 2) {
          ok = step(q, va, vb);
          if (ok && q + 1 < nst) ok = step(q + 1, vb, va);
        }
        if (!ok && lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
      }
      ac += nst;
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(wine_bar + 8 * wb);  // window of this tile no longer read
    }
  } else if (warp == kConvMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t idesc = mma_idesc(C, std::is_same<T, __nv_bfloat16>::value);
      const uint64_t bdesc0 = sw128_desc(base);
      const uint64_t stage_step = stage_bytes >> 4;
      const uint64_t chunk_step = chunk_bytes >> 4;
      // The issuing thread's instruction stream bounds the MMA rate at N <= 128:
      // ring slot and phase advance by compare (no division), descriptors by adds.
      int s = 0;
      uint32_t ph = 0;
      int j = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
        const int ab = j & 1;
        if (ok && !mbar_wait(acce_bar + 8 * ab, ((j >> 1) & 1) ^ 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_ACC);
        }
        tc_fence_after();
        const uint32_t dacc = tmem_base + ab * acc_cols;
        for (int q = 0; q < nst; ++q) {
          const int nc = min(kConvStageChunks, nk - q * kConvStageChunks);
          if (ok && !mbar_wait(full_bar + 8 * s, ph)) {
            ok = false;
            if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_FULL);
          }
          tc_fence_after();
          if (ok) {
            const uint64_t bd = bdesc0 + s * stage_step;
            const uint32_t at = tmem_base + a_col0 + s * (32 * kConvStageChunks);
            tc_mma_f16_ts(dacc, at, bd, idesc, q > 0 ? 1u : 0u);
            tc_mma_f16_ts_acc(dacc, at + 8, bd + 2, idesc);
            tc_mma_f16_ts_acc(dacc, at + 16, bd + 4, idesc);
            tc_mma_f16_ts_acc(dacc, at + 24, bd + 6, idesc);
            if (nc > 1) {
              tc_mma_f16_ts_acc(dacc, at + 32, bd + chunk_step, idesc);
              tc_mma_f16_ts_acc(dacc, at + 40, bd + chunk_step + 2, idesc);
              tc_mma_f16_ts_acc(dacc, at + 48, bd + chunk_step + 4, idesc);
              tc_mma_f16_ts_acc(dacc, at + 56, bd + chunk_step + 6, idesc);
            }
          }
          tc_commit(empty_bar + 8 * s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        tc_commit(accf_bar + 8 * ab);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int half = warp >> 2;
    const int bar_id = 3 + quad;
    float4* xch = xch_all + quad * 64;
    {
      float* lnaw = vecs + 1024;
      for (int i = tid; i < C; i += kEpiWarps * 32) {
        vecs[i] = __ldg(a.bias + i);
        lnaw[i] = a.ln_a_w ? __ldg(a.ln_a_w + i) : 0.f;
        lnaw[256 + i] = a.ln_a_b ? __ldg(a.ln_a_b + i) : 0.f;
        lnaw[512 + i] = a.ln_b_w ? __ldg(a.ln_b_w + i) : 0.f;
        lnaw[768 + i] = a.ln_b_b ? __ldg(a.ln_b_b + i) : 0.f;
        lnaw[1024 + i] = a.gamma ? __ldg(a.gamma + i) : 0.f;
        lnaw[1280 + i] = a.head_w ? __ldg(a.head_w + i) : 0.f;
      }
      asm volatile("bar.sync 2, %0;\n" ::"n"(kEpiWarps * 32) : "memory");
    }
    const EpiVecs ev{vecs, vecs + 1024, vecs + 1024 + 256, vecs + 1024 + 512, vecs + 1024 + 768,
                     vecs + 1024 + 1024, vecs + 1024 + 1280};
    // this thread's row context for tile t (position-block row mapping)
    const int r_in = quad * 32 + lane;
    const int rp = r_in / lpb, ri = r_in - rp * lpb;
    auto conv_row = [&](int t) {
      EpiRow er;
      const int pos = t * geo.ppt + rp;
      const int m = pos * geo.cells + ri;
      er.valid = ri < geo.cells && pos < geo.npos && m < a.M;
      er.mc = er.valid ? m : a.M - 1;
      er.orow = a.orow_from_gidx ? (long long)__ldg(a.gidx + (long long)er.mc * TAPS) : (long long)er.mc;
      er.mk = ((a.flags & (EPI_MASK | EPI_HEAD)) && a.rowmask) ? __ldg(a.rowmask + er.orow) : 1.f;
      er.lnb_row = (a.flags & EPI_LN_B) != 0;
      if (a.flags & EPI_LNB_TOKENS) er.lnb_row = er.lnb_row && er.valid && (er.orow % a.seq_len) < a.ntok;
      return er;
    };
    // quadrant -> (position, first cell) for the TMA boxes
    const int qp = (quad * 32) / lpb, qi0 = quad * 32 - qp * lpb;
    uint32_t rphase = 0;
    int j = 0;
    EpiRow row = conv_row(blockIdx.x);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int ab = j & 1;
      const EpiRow row_next = conv_row(t + gridDim.x);  // loads in flight during this tile
      // rows of this quadrant: cells [qi0, qi0 + 32) of position t * ppt + qp, i.e. rows
      // tokoff + qi0 ... of that position's block (the 3D maps clip past its end)
      // (a 16-bit residual, EPI_RES16, comes through the map passed in the fp32 slot)
      const EpiTma etma{&tmap_o16, &tmap_o32, &tmap_o32, gbase + stg_off + warp * 6144,
                        gbase + stg_off + warp * 6144 + 4096, rload_bar + 8 * warp, t * geo.ppt + qp,
                        (a.flags & EPI_RES16) ? &tmap_o32 : nullptr};
      // the residual rows of the first chunk are requested before the
      // accumulator is ready, so they arrive during the wait
      const bool pre = HEAVY && ok && (a.flags & EPI_RESID);
      if (pre) epi_request_resid(etma, half * (C >> 1), geo.tokoff + qi0, lane);
      const bool got = ok && mbar_wait_sleep(accf_bar + 8 * ab, (j >> 1) & 1);
      ok = __all_sync(0xffffffffu, got) != 0;
      ok = bar_red_and(bar_id, 64, ok);
      if (!ok && lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_EPILOGUE);
      tc_fence_after();
      if (!ok && pre) epi_drain_resid(etma, rphase);
      if (ok) {
        const uint32_t trow = tmem_base + ab * acc_cols + ((uint32_t)(quad * 32) << 16);
        if constexpr (HEAVY) {
          epilogue_tile_tma<T, HEAVY, TAPS == 19>(a, ev, etma, rphase, ok, xch, bar_id, half, row, geo.tokoff + qi0,
                                                  0, trow, lane, pre);
        } else {
          epilogue_tile<T, HEAVY>(a, ev, xch, bar_id, half, row, 0, trow, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar + 8 * ab);
      row = row_next;
    }
    if (HEAVY && lane == 0) bulk_wait_all();  // the staging stays valid until the stores completed
    __syncwarp();
  }

  if (!ok && a.err) atomicOr(a.err, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == kConvMmaWarp) tmem_dealloc(tmem_base, ncols);
}

}  // namespace sb
