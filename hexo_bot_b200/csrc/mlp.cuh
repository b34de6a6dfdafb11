// The attention block's MLP in one kernel (model.py:508-514, AttnBlock's
// `x + ls_mlp(fc2(gelu(fc1(ln2(x)))))`), followed by the LayerNorm of
// whatever reads the stream next:
//
//   h      = GELU(X @ W1^T + b1)                  X = LN2 rows (16-bit), h: 2C wide
//   stream = stream + gamma * mask * (h @ W2^T + b2)   (fp32 residual stream, in place)
//   out16  = LN_b(stream)                          (all rows, or token rows only)
//
// The hidden activations never leave the SM: fc1 accumulates in TMEM, the
// GELU pass turns the accumulator into 16-bit pairs in the same TMEM columns,
// and fc2 reads them back as its A operand (tcgen05 TS form). Compared with
// two GEMM launches this saves the 2C-wide hidden row's HBM write and read
// (4C bytes + 4C bytes per row).
//
// Both weight matrices stay resident in shared memory for the whole
// persistent kernel. TMEM holds two tile buffers of 2C columns each; buffer b
// is [h | acc2]: the GELU pass writes h over the first C columns of the fc1
// accumulator (it reads each 32-column chunk before anything is written over
// it), and fc2 accumulates into the last C columns after the whole fc1
// accumulator has been read.
//
// Warp roles (320 threads):
//   warps 0-3  tile group 0 (even tiles of this CTA), one warp per TMEM lane
//              quadrant: GELU pass, then the residual / LayerNorm epilogue
//   warps 4-7  tile group 1 (odd tiles), the same on TMEM buffer 1
//   warp 8     MMA issue (one thread): fc1 of two tiles, then fc2 of both
//   warp 9     TMA producer: both weight matrices once, then one X tile at a
//              time (single buffer, refilled as soon as fc1 has read it)
// Every mbarrier wait is bounded; a timeout sets a status bit and unwinds.
#pragma once

#include "gemm.cuh"

namespace sb {

struct MlpArgs {
  const void* X;          // [M][C] 16-bit rows (LayerNorm 2 of the stream)
  int M;                  // rows
  int C;                  // channels: 64 or 128 (hidden 2C)
  const float* b1;        // [2C]
  const float* b2;        // [C]
  const float* gamma;     // [C] layer scale
  const float* rowmask;   // [M] 0 / 1
  const float* ln_b_w;    // [C] LayerNorm applied to the updated stream
  const float* ln_b_b;
  float eps;
  int lnb_tokens;         // 1: LayerNorm only on token rows (row % seq_len < ntok), raw stream elsewhere
  int seq_len;
  int ntok;
  int* err;
};

constexpr int kMlpMmaWarp = 8;
constexpr int kMlpProducerWarp = 9;
constexpr int kMlpThreads = 320;

__host__ __device__ constexpr int mlp_w1_bytes(int c) { return (c / 64) * (2 * c) * 128; }
__host__ __device__ constexpr int mlp_w2_bytes(int c) { return (2 * c / 64) * c * 128; }
__host__ __device__ constexpr int mlp_x_bytes(int c) { return (c / 64) * kBlockM * 128; }
__host__ __device__ constexpr int mlp_smem_bytes(int c) {
  return 1024 + mlp_w1_bytes(c) + mlp_w2_bytes(c) + mlp_x_bytes(c) + kEpiTmaBytes + 6 * c * 4 + 8 * 24 + 16;
}
static_assert(mlp_smem_bytes(128) <= 227 * 1024, "fused MLP shared memory at C = 128");

// 16 TMEM columns of this thread's row from 16 packed registers.
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&u)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
      "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]),
      "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15])
      : "memory");
}

// L2 prefetch of `bytes` (a multiple of 16) starting at a 16-byte aligned address.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kMlpThreads, 1)
    mlp_kernel(const MlpArgs a, const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w1,
               const __grid_constant__ CUtensorMap tmap_w2, const __grid_constant__ CUtensorMap tmap_o16,
               const __grid_constant__ CUtensorMap tmap_o32, float* out32) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int C = a.C;
  const int H = 2 * C;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t w1_off = 0;
  const uint32_t w2_off = w1_off + mlp_w1_bytes(C);
  const uint32_t x_off = w2_off + mlp_w2_bytes(C);
  const uint32_t stg_off = x_off + mlp_x_bytes(C);  // 1024-aligned: every block above is
  const uint32_t vec_off = stg_off + kEpiTmaBytes;
  float* vb1 = reinterpret_cast<float*>(gbase + vec_off);  // [2C]
  float* vb2 = vb1 + H;                                    // [C]
  float* vgam = vb2 + C;
  float* vlnw = vgam + C;
  float* vlnb = vlnw + C;
  const uint32_t bar0 = base + vec_off + 6 * C * 4;
  const uint32_t wfull_bar = bar0;
  const uint32_t xfull_bar = bar0 + 8;
  const uint32_t xempty_bar = bar0 + 16;
  const uint32_t accf1_bar = bar0 + 24;   // [2] fc1 accumulator of buffer b complete
  const uint32_t hfull_bar = bar0 + 40;   // [2] h of buffer b written (4 warps)
  const uint32_t accf2_bar = bar0 + 56;   // [2] fc2 accumulator complete
  const uint32_t bufe_bar = bar0 + 72;    // [2] buffer b read by the epilogue (4 warps)
  const uint32_t rload_bar = bar0 + 88;   // [8] residual loads, one per epilogue warp
  const uint32_t tmem_slot = bar0 + 152;
  volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const int tiles = (a.M + kBlockM - 1) / kBlockM;
  const int ntile = (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  pdl_launch_dependents();
  if (warp == kMlpMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(wfull_bar, 1);
    mbar_init(xfull_bar, 1);
    mbar_init(xempty_bar, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf1_bar + 8 * i, 1);
      mbar_init(hfull_bar + 8 * i, 4);
      mbar_init(accf2_bar + 8 * i, 1);
      mbar_init(bufe_bar + 8 * i, 4);
    }
    for (int i = 0; i < 8; ++i) mbar_init(rload_bar + 8 * i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w1);
    prefetch_tmap(&tmap_w2);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;
  bool ok = true;

  if (warp == kMlpProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && ntile > 0) {
      // the weights do not depend on the previous kernel
      mbar_arrive_expect_tx(wfull_bar, mlp_w1_bytes(C) + mlp_w2_bytes(C));
      for (int k = 0; k < C / 64; ++k)
        tma_load_2d(base + w1_off + k * H * 128, &tmap_w1, k * 64, 0, wfull_bar);
      for (int k = 0; k < H / 64; ++k)
        tma_load_2d(base + w2_off + k * C * 128, &tmap_w2, k * 64, 0, wfull_bar);
      pdl_wait();
      for (int j = 0; j < ntile; ++j) {
        const int t = blockIdx.x + j * gridDim.x;
        if (!mbar_wait_sleep(xempty_bar, (j & 1) ^ 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
          break;
        }
        mbar_arrive_expect_tx(xfull_bar, mlp_x_bytes(C));
        for (int k = 0; k < C / 64; ++k)
          tma_load_2d(base + x_off + k * kBlockM * 128, &tmap_x, k * 64, t * kBlockM, xfull_bar);
      }
    }
    __syncwarp();
  } else if (warp == kMlpMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0 && ntile > 0) {
      const bool bf = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t idesc1 = mma_idesc(H, bf);
      const uint32_t idesc2 = mma_idesc(C, bf);
      const uint64_t xdesc = sw128_desc(base + x_off);
      const uint64_t w1desc = sw128_desc(base + w1_off);
      const uint64_t w2desc = sw128_desc(base + w2_off);
      const uint64_t xstep = (kBlockM * 128) >> 4;  // one 64-wide K chunk, in descriptor units
      const uint64_t w1step = (uint64_t)(H * 128) >> 4;
      const uint64_t w2step = (uint64_t)(C * 128) >> 4;
      if (!mbar_wait(wfull_bar, 0)) {
        ok = false;
        if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_FULL);
      }
      auto fc1 = [&](int j) {
        const int b = j & 1, k = j >> 1;
        if (ok && !mbar_wait(bufe_bar + 8 * b, (k & 1) ^ 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_ACC);
        }
        if (ok && !mbar_wait(xfull_bar, j & 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_FULL);
        }
        tc_fence_after();
        const uint32_t d = tmem_base + b * H;
        if (ok) {
          for (int kc = 0; kc < C / 64; ++kc) {
            const uint64_t ad = xdesc + kc * xstep, bd = w1desc + kc * w1step;
            tc_mma_f16(d, ad, bd, idesc1, kc > 0 ? 1u : 0u);
            tc_mma_f16_acc(d, ad + 2, bd + 2, idesc1);
            tc_mma_f16_acc(d, ad + 4, bd + 4, idesc1);
            tc_mma_f16_acc(d, ad + 6, bd + 6, idesc1);
          }
        }
        tc_commit(xempty_bar);
        tc_commit(accf1_bar + 8 * b);
      };
      auto fc2 = [&](int j) {
        const int b = j & 1, k = j >> 1;
        if (ok && !mbar_wait(hfull_bar + 8 * b, k & 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_FULL);
        }
        tc_fence_after();
        const uint32_t hcol = tmem_base + b * H;  // h: two 16-bit values per column
        const uint32_t d = hcol + C;
        if (ok) {
          for (int kc = 0; kc < H / 64; ++kc) {
            const uint32_t at = hcol + kc * 32;
            const uint64_t bd = w2desc + kc * w2step;
            tc_mma_f16_ts(d, at, bd, idesc2, kc > 0 ? 1u : 0u);
            tc_mma_f16_ts_acc(d, at + 8, bd + 2, idesc2);
            tc_mma_f16_ts_acc(d, at + 16, bd + 4, idesc2);
            tc_mma_f16_ts_acc(d, at + 24, bd + 6, idesc2);
          }
        }
        tc_commit(accf2_bar + 8 * b);
      };
      // fc1 of a pair of tiles, then fc2 of both: each tile group gets its
      // fc2 as soon as its GELU pass is done, and the next fc1 into a buffer
      // waits only for that buffer's own epilogue.
      for (int j = 0; j < ntile; j += 2) {
        fc1(j);
        if (j + 1 < ntile) fc1(j + 1);
        fc2(j);
        if (j + 1 < ntile) fc2(j + 1);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ tile groups
    const int g = warp >> 2;     // tile group = TMEM buffer
    const int quad = warp & 3;   // TMEM lanes [32 quad, 32 quad + 32)
    for (int i = tid; i < H; i += 256) vb1[i] = __ldg(a.b1 + i);
    for (int i = tid; i < C; i += 256) {
      vb2[i] = __ldg(a.b2 + i);
      vgam[i] = __ldg(a.gamma + i);
      vlnw[i] = __ldg(a.ln_b_w + i);
      vlnb[i] = __ldg(a.ln_b_b + i);
    }
    asm volatile("bar.sync 2, 256;\n" ::: "memory");
    pdl_wait();
    const EpiTma e{&tmap_o16, &tmap_o32, &tmap_o32, gbase + stg_off + warp * 6144, gbase + stg_off + warp * 6144 + 4096,
                   rload_bar + 8 * warp, -1};
    const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + g * H;
    uint32_t rphase = 0;
    int k = 0;
    for (int j = g; j < ntile; j += 2, ++k) {
      const int t = blockIdx.x + j * gridDim.x;
      const int m_first = t * kBlockM + quad * 32;  // row of lane 0
      const int mc = min(m_first + lane, a.M - 1);  // rows past M: clamped, never stored
      // this warp's 32 stream rows are contiguous: bring them into L2 while
      // the GELU pass and fc2 run
      const int nrows = min(32, a.M - m_first);
      if (lane == 0 && nrows > 0) prefetch_l2_bulk(out32 + (long long)m_first * C, (uint32_t)nrows * C * 4);
      const float mk = __ldg(a.rowmask + mc);
      const bool lnb_row = !a.lnb_tokens || (mc % a.seq_len) < a.ntok;
      // the first residual chunk lands while the GELU pass and fc2 run
      const bool pre = ok;
      if (pre) epi_request_resid(e, 0, m_first, lane);

      // ---- GELU pass: fc1 accumulator -> 16-bit h in the same columns
      bool got = ok && mbar_wait_sleep(accf1_bar + 8 * g, k & 1);
      ok = __all_sync(0xffffffffu, got) != 0;
      if (!ok && lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_EPILOGUE);
      tc_fence_after();
      if (ok) {
        for (int c = 0; c < H; c += 32) {
          float v[32], bb[32];
          tmem_ld32(trow + c, v);
          ld_vec<32>(vb1 + c, bb);
          uint32_t u[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            u[i] = MmaTraits<T>::pack(gelu_erf(v[2 * i] + bb[2 * i]), gelu_erf(v[2 * i + 1] + bb[2 * i + 1]));
          tmem_st16u(trow + (c >> 1), u);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(hfull_bar + 8 * g);

      // ---- fc2 epilogue: bias, mask, gamma * (.) + stream, LayerNorm
      got = ok && mbar_wait_sleep(accf2_bar + 8 * g, k & 1);
      ok = __all_sync(0xffffffffu, got) != 0;
      if (!ok && lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_EPILOGUE);
      tc_fence_after();
      if (!ok && pre) epi_drain_resid(e, rphase);
      if (ok) {
        const uint32_t tacc = trow + C;
        float cnt = 0.f, mean = 0.f, m2 = 0.f;
        for (int c = 0; c < C; c += 32) {
          float v[32], x[32];
          stage_reuse(lane);
          if (c > 0) epi_request_resid(e, c, m_first, lane);
          tmem_ld32(tacc + c, v);
          const bool rgot = ok && mbar_wait(e.rbar, rphase);
          ok = __all_sync(0xffffffffu, rgot) != 0;
          rphase ^= 1u;
          unstage_row32(e.st32, lane, x);
          {
            float bb[32], gg[32];
            ld_vec<32>(vb2 + c, bb);
            ld_vec<32>(vgam + c, gg);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = fmaf((v[i] + bb[i]) * mk, gg[i], x[i]);
          }
          stats_merge_w<32>(cnt, mean, m2, v);
          tmem_stw<32>(tacc + c, v);  // parked for the LayerNorm pass
          stage_row32(e.st32, lane, v);
          stage_flush(e, lane, true, e.o32, false, c, m_first);
        }
        const float rstd = rsqrtf(m2 / cnt + a.eps);
        tmem_wait_st();
        for (int c = 0; c < C; c += 32) {
          float v[32], ww[32], bb[32];
          stage_reuse(lane);
          tmem_ld32(tacc + c, v);
          ld_vec<32>(vlnw + c, ww);
          ld_vec<32>(vlnb + c, bb);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = lnb_row ? fmaf((v[i] - mean) * rstd, ww[i], bb[i]) : v[i];
          stage_row16<T>(e.st16, lane, v);
          stage_flush(e, lane, false, nullptr, true, c, m_first);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bufe_bar + 8 * g);
    }
    if (lane == 0) bulk_wait_all();  // the staging stays valid until the stores completed
    __syncwarp();
  }

  if (!ok && a.err) atomicOr(a.err, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == kMlpMmaWarp) tmem_dealloc(tmem_base, 512);
}

}  // namespace sb
