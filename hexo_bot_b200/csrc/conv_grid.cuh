// HexNodeConv (7 taps) over the hex grid itself: the neighbour gather becomes
// a row offset of the tensor-core operand.
//
//   out[m, :] = epilogue( sum_t X[nbr_t(m), :] @ W_t )      (model.py:346-370)
//
// Every cell (q, r) of a position whose cells lie in the radius-4 box is given
// the slot (q + 4) * 10 + (r + 4) of a 10 x 10 block (9 rows of 9 cells, a zero
// tenth column and a zero tenth row); the blocks of consecutive positions
// follow each other. In that layout the neighbour in direction (dq, dr) is the
// slot dq * 10 + dr away for every cell, and every neighbour that is not a
// cell of the position lands on an empty (zero) slot: the tenth column, the
// tenth row, the box corners or the margins. So the conv is
//
//   out[slot] = sum_t window[slot + shift_t] @ W_t
//
// and the A operand of tap t is the window itself, read by the MMA from
// shared memory at a start row shifted by shift_t (tcgen05 descriptors take
// any 128-byte row as start; the 128-byte swizzle follows the absolute
// address). No A operand is built per tap: the only per-tile work besides the
// MMAs is copying each cell row into its slot once (cp.async) and the
// epilogue. Output rows are slots; slots without a cell are not stored.
//
// A position is eligible when every cell is live, lies in the box, owns a
// slot alone, and its neighbour table equals the grid adjacency
// (grid_geom_kernel checks that and sets a batch flag; the forward launches
// this kernel and the windowed conv, and the one the flag does not select
// returns at once).
//
// Tiles are 128 consecutive slots of the concatenated blocks; a job is two
// tiles (one weight stream feeds both accumulators); four TMEM accumulators
// double-buffer jobs against the epilogue.
//
// Warp roles (448 threads): 0-7 epilogue, 8 MMA issue, 9 weight producer,
// 10-13 window producers.
#pragma once

#include "gemm.cuh"

namespace sb {

constexpr int kGridR = 4;
constexpr int kGridW = 2 * kGridR + 2;            // 10 slots per grid row
constexpr int kGridBlock = kGridW * kGridW;       // 100 slots per position
constexpr int kGridMaxCells = (2 * kGridR + 1) * (2 * kGridR + 1);
constexpr int kGridMargin = kGridW;               // largest |shift|
constexpr int kGridWinRows = 2 * kBlockM + 2 * kGridMargin;  // one job's window
__host__ __device__ constexpr int grid_panel_bytes() { return (kGridWinRows * 128 + 1023) / 1024 * 1024; }
constexpr int kGridStages = 4;  // 64 KB of weights in flight
constexpr int kGridWarps = 14;
constexpr int kGridThreads = kGridWarps * 32;
constexpr int kGridMma = 8, kGridWProducer = 9, kGridWin0 = 10;
// Below this many positions per launch the windowed conv alone runs: the grid
// conv's extra launches (geometry check, the kernel the flag skips) cost more
// than it saves when every conv is one or two tiles per SM.
constexpr int kGridMinBatch = 1024;

__host__ __device__ constexpr int conv_grid_smem_bytes(int c) {
  return 1024 + 2 * (c / 64) * grid_panel_bytes() + kGridStages * c * 128 + kEpiSmemBytes +
         8 * (2 * kGridStages + 8) + 16 + kGridWinRows * 4;
}

// slot shift of tap t (tap 0 = the cell, taps 1..6 = DIRECTIONS)
__device__ __forceinline__ int grid_shift(int tap) {
  // DIRECTIONS (1,0) (0,1) (-1,1) (-1,0) (0,-1) (1,-1): dq * W + dr
  switch (tap) {
    case 1: return kGridW;
    case 2: return 1;
    case 3: return 1 - kGridW;
    case 4: return -kGridW;
    case 5: return -1;
    case 6: return kGridW - 1;
    default: return 0;
  }
}

struct GridGeom {
  int npos;                // positions
  int npad;                // cells per position in the inputs
  int S;                   // rows per position in the activation / output layout
  int tokoff;              // rows before the cells in each position's block (8 tokens in the forward)
  const int16_t* slot_cell;  // [npos][100] cell of each slot, -1 = empty
};

// The MMA issue loop of conv_grid_kernel for NBOX 64-channel boxes (C = 64
// NBOX): per job, 7 taps x NBOX boxes of weight stages; each stage feeds 4 K
// steps of the job's two tiles.
template <typename T, int NBOX>
__device__ __forceinline__ void grid_mma_loop(const GemmArgs& a, uint32_t base, uint32_t win_off, uint32_t w_off,
                                              uint32_t wstage, uint32_t panel, uint32_t tmem_base, uint32_t full_bar,
                                              uint32_t empty_bar, uint32_t winf_bar, uint32_t wine_bar,
                                              uint32_t accf_bar, uint32_t acce_bar, int njobs, bool& ok) {
  constexpr int C = NBOX * 64;
  const uint32_t idesc = mma_idesc(C, std::is_same<T, __nv_bfloat16>::value);
  const uint64_t wdesc0 = sw128_desc(base + w_off);
  const uint64_t wstep = wstage >> 4;
  const uint64_t tile_step = (kBlockM * 128) >> 4;  // the job's second tile: 128 rows further
  uint32_t it = 0;
  int i = 0;
  for (int job = blockIdx.x; job < njobs; job += gridDim.x, ++i) {
    const int ab = i & 1, wb = i & 1;
    if (ok && !mbar_wait(acce_bar + 8 * ab, ((i >> 1) & 1) ^ 1)) {
      ok = false;
      if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_ACC);
    }
    if (ok && !mbar_wait(winf_bar + 8 * wb, (i >> 1) & 1)) {
      ok = false;
      if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_FULL);
    }
    tc_fence_after();
    const uint32_t d0 = tmem_base + (2 * ab) * C, d1 = d0 + C;
    const uint64_t adesc0 = sw128_desc(base + win_off + wb * NBOX * panel);
#pragma unroll
    for (int tap = 0; tap < 7; ++tap) {
      const uint64_t arow = (uint64_t)((kGridMargin + grid_shift(tap)) * 128) >> 4;
#pragma unroll
      for (int bx = 0; bx < NBOX; ++bx, ++it) {
        const uint32_t s = it % kGridStages;
        if (ok && !mbar_wait(full_bar + 8 * s, (it / kGridStages) & 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_FULL);
        }
        tc_fence_after();
        if (ok) {
          const uint64_t bd = wdesc0 + s * wstep;
          const uint64_t ad = adesc0 + (uint64_t)(bx * panel >> 4) + arow;
          tc_mma_f16(d0, ad, bd, idesc, (tap | bx) ? 1u : 0u);
          tc_mma_f16_acc(d0, ad + 2, bd + 2, idesc);
          tc_mma_f16_acc(d0, ad + 4, bd + 4, idesc);
          tc_mma_f16_acc(d0, ad + 6, bd + 6, idesc);
          tc_mma_f16(d1, ad + tile_step, bd, idesc, (tap | bx) ? 1u : 0u);
          tc_mma_f16_acc(d1, ad + tile_step + 2, bd + 2, idesc);
          tc_mma_f16_acc(d1, ad + tile_step + 4, bd + 4, idesc);
          tc_mma_f16_acc(d1, ad + tile_step + 6, bd + 6, idesc);
        }
        tc_commit(empty_bar + 8 * s);
      }
    }
    tc_commit(wine_bar + 8 * wb);
    tc_commit(accf_bar + 8 * ab);
  }
}

template <typename T, bool HEAVY>
__global__ void __launch_bounds__(kGridThreads, 1)
    conv_grid_kernel(const GemmArgs a, const GridGeom geo, const __grid_constant__ CUtensorMap tmap_w) {
  // the batch flag selects this kernel or the windowed one (uniform per grid)
  if (a.skip_flag) {
    pdl_wait();
    if (*reinterpret_cast<const volatile int*>(a.skip_flag) == a.skip_value) return;
  }
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int C = a.n_total;  // == a.cin, a multiple of 64
  const int nbox = C / 64;
  const int nk = 7 * nbox;  // 64-wide K chunks: tap-major
  const uint32_t panel = grid_panel_bytes();

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t win_off = 0;                                  // [2][nbox][panel]
  const uint32_t w_off = win_off + 2 * nbox * panel;           // [stages][C rows x 128 B]
  const uint32_t wstage = C * 128;
  const uint32_t epi_off = w_off + kGridStages * wstage;
  float* vecs = reinterpret_cast<float*>(gbase + epi_off);
  float4* xch_all = reinterpret_cast<float4*>(gbase + epi_off + kEpiVecFloats * 4);
  const uint32_t bar0 = base + epi_off + kEpiSmemBytes;
  const uint32_t full_bar = bar0;                           // [stages] weight stage landed
  const uint32_t empty_bar = full_bar + 8 * kGridStages;    // [stages] weight stage consumed
  const uint32_t winf_bar = empty_bar + 8 * kGridStages;    // [2] window written
  const uint32_t wine_bar = winf_bar + 16;          // [2] window consumed
  const uint32_t accf_bar = wine_bar + 16;          // [2] accumulator pair ready
  const uint32_t acce_bar = accf_bar + 16;          // [2] accumulator pair drained
  const uint32_t tmem_slot = acce_bar + 16;
  volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));
  // source row of every window row of the job being filled (-1 = zero row)
  int* win_src = reinterpret_cast<int*>(gbase + (tmem_slot - base) + 16);

  const long long nslots = (long long)geo.npos * kGridBlock;
  const int ntiles = (int)((nslots + kBlockM - 1) / kBlockM);
  const int njobs = (ntiles + 1) / 2;

  pdl_launch_dependents();
  if (warp == kGridMma) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kGridStages; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(empty_bar + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(winf_bar + 8 * i, 128);
      mbar_init(wine_bar + 8 * i, 1);
      mbar_init(accf_bar + 8 * i, 1);
      mbar_init(acce_bar + 8 * i, kEpiWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    prefetch_tmap(&tmap_w);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;
  bool ok = true;
  if (warp != kGridWProducer && warp != kGridMma) pdl_wait();

  if (warp >= kGridWin0) {
    // ------------------------------------------------------------ window producers
    // each cell row into its slot (zeros for empty slots), 128-byte swizzle
    const int ptid = tid - kGridWin0 * 32;
    const T* X = reinterpret_cast<const T*>(a.A);
    int i = 0;
    for (int job = blockIdx.x; job < njobs; job += gridDim.x, ++i) {
      const int wb = i & 1;
      bool free_ok = ok && mbar_wait_sleep(wine_bar + 8 * wb, ((i >> 1) & 1) ^ 1);
      free_ok = bar_red_and(1, 128, free_ok);  // the four producer warps decide together
      if (!free_ok) {
        ok = false;
        if (a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
        break;
      }
      const long long g0 = (long long)job * 2 * kBlockM - kGridMargin;  // slot of window row 0
      const uint32_t wbase = base + win_off + wb * nbox * panel;
      // 1) the source row of each window row: independent loads, all in flight
      for (int row = ptid; row < kGridWinRows; row += 128) {
        const long long gs = g0 + row;
        int src = -1;
        if (gs >= 0 && gs < nslots) {
          const long long b = gs / kGridBlock;
          const int cell = __ldg(geo.slot_cell + gs);
          src = cell >= 0 ? (int)(b * geo.S + geo.tokoff + cell) : -1;
        }
        win_src[row] = src;
      }
      asm volatile("bar.sync 1, 128;\n" ::: "memory");
      // 2) the copies: thread p takes 16-byte piece p % 8 of rows p / 8, p / 8 + 16, ...
      {
        const int piece = ptid & 7;
        const uint32_t pbase = wbase + (piece << 4);
        for (int row = ptid >> 3; row < kGridWinRows; row += 16) {
          const int src = win_src[row];
          const bool live = src >= 0;
          const T* p = live ? X + ((long long)src * C + piece * 8) : X;
          const uint32_t dst = pbase + row * 128;
          const uint32_t swz = (uint32_t)(((piece ^ (row & 7)) - piece) << 4);  // swizzled piece offset delta
          cp_async16(dst + swz, p, live ? 16u : 0u);
          if (nbox == 2) cp_async16(dst + panel + swz, live ? p + 64 : X, live ? 16u : 0u);
        }
      }
      asm volatile("bar.sync 1, 128;\n" ::: "memory");  // win_src may be refilled for the next job
      cp_async_commit();
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(winf_bar + 8 * wb);
    }
  } else if (warp == kGridWProducer) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int job = blockIdx.x; job < njobs; job += gridDim.x) {
        for (int c = 0; c < nk; ++c, ++it) {
          const int s = it % kGridStages;
          if (ok && !mbar_wait_sleep(empty_bar + 8 * s, ((it / kGridStages) & 1) ^ 1)) {
            ok = false;
            if (a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
          }
          if (!ok) break;
          mbar_arrive_expect_tx(full_bar + 8 * s, wstage);
          tma_load_2d(base + w_off + s * wstage, &tmap_w, c * kChunkK, 0, full_bar + 8 * s);
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == kGridMma) {
    // ------------------------------------------------------------ MMA issue
    // One thread issues every MMA; its instruction stream is the limit at
    // N = 128 (an MMA takes ~64 tensor cycles), so the loop is fully unrolled
    // over (tap, channel box) with descriptors formed by constant adds.
    if (lane == 0) {
      if (nbox == 2)
        grid_mma_loop<T, 2>(a, base, win_off, w_off, wstage, panel, tmem_base, full_bar, empty_bar, winf_bar,
                            wine_bar, accf_bar, acce_bar, njobs, ok);
      else
        grid_mma_loop<T, 1>(a, base, win_off, w_off, wstage, panel, tmem_base, full_bar, empty_bar, winf_bar,
                            wine_bar, accf_bar, acce_bar, njobs, ok);
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
      for (int k = tid; k < C; k += kEpiWarps * 32) {
        vecs[k] = __ldg(a.bias + k);
        lnaw[k] = a.ln_a_w ? __ldg(a.ln_a_w + k) : 0.f;
        lnaw[256 + k] = a.ln_a_b ? __ldg(a.ln_a_b + k) : 0.f;
        lnaw[512 + k] = a.ln_b_w ? __ldg(a.ln_b_w + k) : 0.f;
        lnaw[768 + k] = a.ln_b_b ? __ldg(a.ln_b_b + k) : 0.f;
        lnaw[1024 + k] = a.gamma ? __ldg(a.gamma + k) : 0.f;
        lnaw[1280 + k] = a.head_w ? __ldg(a.head_w + k) : 0.f;
      }
      asm volatile("bar.sync 2, %0;\n" ::"n"(kEpiWarps * 32) : "memory");
    }
    const EpiVecs ev{vecs, vecs + 1024, vecs + 1024 + 256, vecs + 1024 + 512, vecs + 1024 + 768,
                     vecs + 1024 + 1024, vecs + 1024 + 1280};
    const int r_in = quad * 32 + lane;
    const bool use_mask = ((a.flags & (EPI_MASK | EPI_HEAD)) != 0) && a.rowmask;
    auto slot_of = [&](int t) { return (long long)t * kBlockM + r_in; };
    // output row context of slot row r_in of tile t (cell, row mask), loaded
    // one job ahead so the latency hides behind the current job
    struct Pre { int cell; float mk; };
    auto pre_of = [&](int t) -> Pre {
      const long long gs = slot_of(t);
      Pre p{-1, 0.f};
      if (t < ntiles && gs < nslots) {
        p.cell = __ldg(geo.slot_cell + gs);
        if (p.cell >= 0)
          p.mk = use_mask ? __ldg(a.rowmask + (gs / kGridBlock) * geo.S + geo.tokoff + p.cell) : 1.f;
      }
      return p;
    };
    auto grid_row = [&](int t, Pre p) {
      EpiRow er;
      const long long b = slot_of(t) / kGridBlock;
      er.valid = p.cell >= 0;
      er.mc = er.valid ? (int)(b * geo.npad + p.cell) : 0;
      er.orow = er.valid ? b * geo.S + geo.tokoff + p.cell : 0;
      er.mk = p.mk;
      er.lnb_row = (a.flags & EPI_LN_B) != 0 && !(a.flags & EPI_LNB_TOKENS);
      return er;
    };
    int i = 0;
    Pre c0 = pre_of(2 * blockIdx.x), c1 = pre_of(2 * blockIdx.x + 1);
    for (int job = blockIdx.x; job < njobs; job += gridDim.x, ++i) {
      const int ab = i & 1;
      const Pre cur0 = c0, cur1 = c1;
      c0 = pre_of(2 * (job + gridDim.x));  // next job's rows, in flight during this one
      c1 = pre_of(2 * (job + gridDim.x) + 1);
      EpiRow row = grid_row(2 * job, cur0);
      const bool got = ok && mbar_wait_sleep(accf_bar + 8 * ab, (i >> 1) & 1);
      ok = __all_sync(0xffffffffu, got) != 0;
      ok = bar_red_and(bar_id, 64, ok);
      if (!ok && lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_EPILOGUE);
      tc_fence_after();
      if (ok) {
        for (int u = 0; u < 2; ++u) {
          if (u == 1) row = grid_row(2 * job + 1, cur1);
          const uint32_t trow = tmem_base + (2 * ab + u) * C + ((uint32_t)(quad * 32) << 16);
          epilogue_tile<T, HEAVY>(a, ev, xch, bar_id, half, row, 0, trow, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar + 8 * ab);
    }
  }

  if (!ok && a.err) atomicOr(a.err, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == kGridMma) tmem_dealloc(tmem_base, 512);
}

// Grid slots of every position and the batch flag: flag = 1 when every
// position is eligible for conv_grid_kernel (every cell live, in the radius-4
// box, alone in its slot, and its six gather rows equal to the cells at the
// grid neighbours). One warp per position; the flag starts at 1 (set by the
// input staging kernel) and any ineligible position clears it.
__global__ void grid_geom_kernel(const int32_t* coords32, const int32_t* gidx, const float* rowmask, int B, int npad,
                                 int S, int16_t* slot_cell, int* flag) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int16_t owner_s[8][kGridBlock];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + w;
  if (b >= B) return;
  int16_t* owner = owner_s[w];
  for (int s = lane; s < kGridBlock; s += 32) owner[s] = -1;
  __syncwarp();
  bool good = npad <= kGridMaxCells;
  for (int n = lane; n < npad && good; n += 32) {
    const int q = coords32[((long long)b * npad + n) * 2], r = coords32[((long long)b * npad + n) * 2 + 1];
    const bool live = rowmask[(long long)b * S + kNumTok + n] != 0.f;
    const bool in = q >= -kGridR && q <= kGridR && r >= -kGridR && r <= kGridR;
    if (!live || !in) {
      good = false;
    } else {
      const int s = (q + kGridR) * kGridW + (r + kGridR);
      // 16-bit slots: claim with a 32-bit CAS on the aligned pair
      uint32_t* word = reinterpret_cast<uint32_t*>(owner + (s & ~1));
      const int shiftb = (s & 1) * 16;
      uint32_t old = *reinterpret_cast<volatile uint32_t*>(word);
      while (true) {
        if (((old >> shiftb) & 0xFFFFu) != 0xFFFFu) { good = false; break; }
        const uint32_t nv = (old & ~(0xFFFFu << shiftb)) | ((uint32_t)n << shiftb);
        const uint32_t prev = atomicCAS(word, old, nv);
        if (prev == old) break;
        old = prev;
      }
    }
  }
  good = __all_sync(0xffffffffu, good) != 0;
  __syncwarp();
  if (good) {
    for (int n = lane; n < npad; n += 32) {
      const int q = coords32[((long long)b * npad + n) * 2], r = coords32[((long long)b * npad + n) * 2 + 1];
      const int s = (q + kGridR) * kGridW + (r + kGridR);
      for (int k = 1; k < 7; ++k) {
        const int t = s + grid_shift(k);
        const int want = (t >= 0 && t < kGridBlock) ? owner[t] : -1;
        const int g = gidx[((long long)b * npad + n) * 7 + k];
        const int got = g < 0 ? -1 : g - (b * S + kNumTok);
        if (want != got) good = false;
      }
    }
    good = __all_sync(0xffffffffu, good) != 0;
  }
  for (int s = lane; s < kGridBlock; s += 32) slot_cell[(long long)b * kGridBlock + s] = good ? owner[s] : -1;
  if (!good && lane == 0) atomicAnd(flag, 0);
}

// The op-level hex_conv's tables from its row-local gather table (B, npad, 7)
// (tap 0 = the cell, missing = npad) and u8 mask: absolute gather rows
// (-1 = missing), the float row mask, and the grid slots, found from the
// gather table alone (the op has no coordinates): a search places cell 0 at
// (0, 0) and the neighbour of a placed cell in direction D_k at its offset
// +D_k, then shifts the placement into the box. A position is eligible when
// every cell is placed, the placement fits 9 x 9, slots are unique, and every
// gather row equals the cell at the grid neighbour. One warp per position;
// an ineligible position sets *flag (zeroed beforehand).
__global__ void grid_embed_kernel(const int32_t* local, const uint8_t* mask, int B, int npad, int32_t* gabs,
                                  float* rowmask, int16_t* slot_cell, int* flag) {
  __shared__ int8_t qs[8][kGridMaxCells], rs[8][kGridMaxCells];
  __shared__ int16_t owner_s[8][kGridBlock];
  __shared__ int16_t nb_s[8][kGridMaxCells][6];  // row-local neighbours, -1 = missing
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + w;
  if (b >= B) return;
  int8_t* q = qs[w];
  int8_t* r = rs[w];
  int16_t* owner = owner_s[w];
  int16_t(*nb)[6] = nb_s[w];
  const int dq[7] = {0, 1, 0, -1, -1, 0, 1}, dr[7] = {0, 0, 1, 1, 0, -1, -1};
  const long long row0 = (long long)b * npad;
  // the op's tables: absolute gather rows (missing = -1) and the float row mask
  for (int i = lane; i < npad * 7; i += 32) {
    const int v = local[row0 * 7 + i];
    gabs[row0 * 7 + i] = (v >= 0 && v < npad) ? (int32_t)(row0 + v) : -1;
  }
  for (int n = lane; n < npad; n += 32) rowmask[row0 + n] = mask[row0 + n] ? 1.f : 0.f;
  bool good = npad <= kGridMaxCells;
  if (good) {
    // the position's neighbours into shared memory (all loads in flight at once)
    for (int i = lane; i < npad * 6; i += 32) {
      const int n = i / 6, k = i - n * 6;
      const int v = local[(row0 + n) * 7 + 1 + k];
      const bool self = local[(row0 + n) * 7] == n;
      nb[n][k] = (int16_t)((v >= 0 && v < npad && self) ? v : (v >= npad || v < 0 ? -1 : -2));
    }
    for (int n = lane; n < npad; n += 32) q[n] = r[n] = 127;
    for (int s = lane; s < kGridBlock; s += 32) owner[s] = -1;
    __syncwarp();
    if (lane == 0) q[0] = r[0] = 0;
    __syncwarp();
    // placement: grow from cell 0 along the gather table
    for (int round = 0; round < npad; ++round) {
      bool changed = false;
      for (int n = lane; n < npad; n += 32) {
        const int qn = q[n], rn = r[n];
        if (qn == 127) continue;
        for (int k = 1; k < 7; ++k) {
          const int j = nb[n][k - 1];
          if (j >= 0 && q[j] == 127) {
            q[j] = (int8_t)max(-100, min(100, qn + dq[k]));
            r[j] = (int8_t)max(-100, min(100, rn + dr[k]));
            changed = true;
          }
        }
      }
      __syncwarp();
      if (!__any_sync(0xffffffffu, changed)) break;
    }
    int mnq = 127, mxq = -127, mnr = 127, mxr = -127;
    for (int n = lane; n < npad; n += 32) {
      if (q[n] == 127) good = false;
      mnq = min(mnq, (int)q[n]); mxq = max(mxq, (int)q[n]);
      mnr = min(mnr, (int)r[n]); mxr = max(mxr, (int)r[n]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mnq = min(mnq, __shfl_xor_sync(0xffffffffu, mnq, o));
      mxq = max(mxq, __shfl_xor_sync(0xffffffffu, mxq, o));
      mnr = min(mnr, __shfl_xor_sync(0xffffffffu, mnr, o));
      mxr = max(mxr, __shfl_xor_sync(0xffffffffu, mxr, o));
    }
    good = __all_sync(0xffffffffu, good) && mxq - mnq <= 2 * kGridR && mxr - mnr <= 2 * kGridR;
    if (good) {
      for (int n = lane; n < npad; n += 32) {
        const int s = (q[n] - mnq) * kGridW + (r[n] - mnr);
        uint32_t* word = reinterpret_cast<uint32_t*>(owner + (s & ~1));
        const int shiftb = (s & 1) * 16;
        uint32_t old = *reinterpret_cast<volatile uint32_t*>(word);
        while (true) {
          if (((old >> shiftb) & 0xFFFFu) != 0xFFFFu) { good = false; break; }
          const uint32_t nv = (old & ~(0xFFFFu << shiftb)) | ((uint32_t)n << shiftb);
          const uint32_t prev = atomicCAS(word, old, nv);
          if (prev == old) break;
          old = prev;
        }
      }
      good = __all_sync(0xffffffffu, good);
      __syncwarp();
    }
    if (good) {
      // every gather row must be the cell at the grid neighbour (missing = empty)
      for (int n = lane; n < npad; n += 32) {
        const int s = (q[n] - mnq) * kGridW + (r[n] - mnr);
        for (int k = 1; k < 7; ++k) {
          const int t = s + grid_shift(k);
          const int want = (t >= 0 && t < kGridBlock) ? owner[t] : -1;
          if (want != nb[n][k - 1]) good = false;
        }
      }
      good = __all_sync(0xffffffffu, good);
    }
  }
  for (int s = lane; s < kGridBlock; s += 32) slot_cell[(long long)b * kGridBlock + s] = good ? owner[s] : -1;
  if (!good && lane == 0) atomicOr(flag, 1);
}

}  // namespace sb
