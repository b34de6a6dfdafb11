// Gather-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), with the
// Shrimp epilogues fused in.
//
//   acc[m, n] = sum_t sum_c  X[src(m, t), c] * W[n, t*Cin + c]
//
// where src(m, t) = gidx[m*T + t] (a gathered row, -1 = zero row) or m when no
// gather table is given. This single kernel covers HexNodeConv (T = 7 taps:
// self + 6 neighbours; model.py:346-370), the 19-tap ray microbench and every
// nn.Linear of the attention block (T = 1).
//
// One CTA = 128 output rows x BN columns (BN <= 256, multiple of 16). Four
// warps load A (gathered rows) and B (weights) into a multi-stage ring of
// 128-byte-swizzled K-major shared-memory tiles with cp.async (zero-fill for
// missing neighbours); one thread issues tcgen05.mma (M=128, N=BN, K=16) into a
// TMEM fp32 accumulator and commits each stage to an mbarrier that releases
// the stage for refill. The epilogue gives each thread one accumulator row
// (TMEM lane = row), so LayerNorm statistics need no cross-thread reduction.
#pragma once

#include <type_traits>

#include "ptx.cuh"

namespace sb {

enum EpiFlags : int {
  EPI_LN_A = 1 << 0,        // v = LayerNorm_a(acc + bias)
  EPI_RELU = 1 << 1,        // relu after LN_a
  EPI_GELU = 1 << 2,        // erf-GELU after LN_a
  EPI_MASK = 1 << 3,        // v *= rowmask[out_row]
  EPI_RESID = 1 << 4,       // v = out32[out_row] + gamma * v (in place)
  EPI_POST_RELU = 1 << 5,   // relu after the residual add
  EPI_OUT32 = 1 << 6,       // write v (fp32) to out32[out_row]
  EPI_OUT16 = 1 << 7,       // write v (16-bit) to out16[out_row] (or LN_b(v), see below)
  EPI_LN_B = 1 << 8,        // out16 = LayerNorm_b(v) (v re-read from out32)
  EPI_LNB_TOKENS = 1 << 9,  // LN_b only on token rows (out_row % seq_len < ntok); others raw
  EPI_OUT32B = 1 << 10,     // also write LayerNorm_b(v) in fp32 to out32b
  EPI_HEAD = 1 << 11,       // head_out[m] = rowmask * (sum_c relu(v_c) head_w[c] + head_b)
  EPI_RES16 = 1 << 12,      // v = relu(v + res16[out_row]) (ray-conv microbench)
};

struct GemmArgs {
  // A operand: rows of a 16-bit row-major matrix.
  const void* A;
  long long lda;           // elements between consecutive source rows
  int cin;                 // channels per tap (multiple of 8)
  int taps;                // T
  const int32_t* gidx;     // [M][T] source rows, -1 = zero; nullptr = identity (T == 1)
  int M;                   // output rows
  // B operand: [n_total][kpad] K-major 16-bit weights, kpad multiple of 64.
  const void* Bw;
  int kpad;
  int n_total;
  int bn;                  // N tile (multiple of 16, <= 256)
  // epilogue
  int flags;
  const float* bias;       // [n_total]
  const float* ln_a_w;
  const float* ln_a_b;
  const float* ln_b_w;
  const float* ln_b_b;
  float eps;
  const float* rowmask;    // per output row (0/1)
  const float* gamma;      // [N]
  float* out32;            // fp32 rows, row stride ld32
  long long ld32;
  float* out32b;
  long long ld32b;
  void* out16;             // 16-bit rows, row stride ld16
  long long ld16;
  const void* res16;       // 16-bit residual rows (microbench)
  long long ldr16;
  const float* head_w;
  float head_b;
  float* head_out;
  int seq_len;             // rows per position in the seq layout (for EPI_LNB_TOKENS)
  int ntok;
  int* err;                // device status word
};

constexpr int kGemmThreads = 128;
constexpr int kBlockM = 128;
constexpr int kChunkK = 64;        // 64 x 16-bit = one 128-byte swizzle row
constexpr int kTileABytes = kBlockM * 128;

__host__ __device__ constexpr int gemm_stage_bytes(int bn) { return kTileABytes + bn * 128; }
__host__ __device__ constexpr int gemm_smem_bytes(int bn, int stages) {
  return 1024 /*align slack*/ + stages * gemm_stage_bytes(bn) + 256 /*barriers + tmem slot*/;
}

template <typename T>
__device__ __forceinline__ void load16(const void* base, long long off, float (&v)[16]) {
  const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(base) + off);
  uint4 u0 = p[0], u1 = p[1];
  const T* h0 = reinterpret_cast<const T*>(&u0);
  const T* h1 = reinterpret_cast<const T*>(&u1);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = to_f32<T>(h0[i]);
    v[8 + i] = to_f32<T>(h1[i]);
  }
}

template <typename T>
__device__ __forceinline__ void store16(void* base, long long off, const float (&v)[16]) {
  uint4 u0, u1;
  T* h0 = reinterpret_cast<T*>(&u0);
  T* h1 = reinterpret_cast<T*>(&u1);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h0[i] = from_f32<T>(v[i]);
    h1[i] = from_f32<T>(v[8 + i]);
  }
  uint4* p = reinterpret_cast<uint4*>(reinterpret_cast<T*>(base) + off);
  p[0] = u0;
  p[1] = u1;
}

__device__ __forceinline__ void store16_f32(float* p, const float (&v)[16]) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

__device__ __forceinline__ void load16_f32(const float* p, float (&v)[16]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 f = q[i];
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}

// Chan's merge of a 16-value chunk into running (count, mean, M2).
__device__ __forceinline__ void stats_merge(float& cnt, float& mean, float& m2, const float (&v)[16]) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) s += v[i];
  const float cm = s * (1.f / 16.f);
  float c2 = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float d = v[i] - cm;
    c2 = fmaf(d, d, c2);
  }
  const float tot = cnt + 16.f;
  const float delta = cm - mean;
  mean = fmaf(delta, 16.f / tot, mean);
  m2 += c2 + delta * delta * (cnt * 16.f / tot);
  cnt = tot;
}

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }

// Issue the cp.async copies of K-chunk `chunk` for this CTA's tile into stage
// buffers sA / sB (shared addresses).
template <typename T>
__device__ __forceinline__ void gemm_load_chunk(const GemmArgs& a, int m0, int n0, int chunk, uint32_t sA,
                                                uint32_t sB, int tid) {
  const int kbase = chunk * kChunkK;
  const int p = tid & 7;          // 16-byte piece within the 128-byte row
  const int rsub = tid >> 3;      // 0..15
  const int k = kbase + p * 8;
  const int ktot = a.taps * a.cin;
  const int tap = k / a.cin;
  const int ch = k - tap * a.cin;
  const T* X = reinterpret_cast<const T*>(a.A);
#pragma unroll
  for (int i = 0; i < kBlockM / 16; ++i) {
    const int r = rsub + 16 * i;
    const int m = m0 + r;
    long long src_row = -1;
    if (m < a.M && k < ktot) src_row = a.gidx ? (long long)__ldg(a.gidx + (long long)m * a.taps + tap) : m;
    const void* src = X;
    uint32_t bytes = 0;
    if (src_row >= 0) {
      src = X + src_row * a.lda + ch;
      bytes = 16;
    }
    cp_async16(sA + r * 128 + ((p ^ (r & 7)) << 4), src, bytes);
  }
  const T* W = reinterpret_cast<const T*>(a.Bw);
  for (int r = rsub; r < a.bn; r += 16) {
    const int n = n0 + r;
    const void* src = W;
    uint32_t bytes = 0;
    if (n < a.n_total) {
      src = W + (long long)n * a.kpad + kbase + p * 8;
      bytes = 16;
    }
    cp_async16(sB + r * 128 + ((p ^ (r & 7)) << 4), src, bytes);
  }
}

template <typename T, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  static_assert(STAGES >= 3, "need >= 3 stages");
  constexpr int PF = STAGES - 2;  // chunks prefetched ahead
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int m0 = blockIdx.x * kBlockM;
  const int n0 = blockIdx.y * a.bn;

  // 1024-byte aligned stage ring (the 128-byte swizzle pattern is anchored to
  // 1024-byte boundaries).
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t stage_bytes = kTileABytes + a.bn * 128;
  const uint32_t bar_base = base + STAGES * stage_bytes;   // STAGES mbarriers (8 B each)
  const uint32_t tmem_slot = bar_base + 8 * STAGES;
  uint8_t* smem_gen = smem_raw + (base - smem_u32(smem_raw));
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(smem_gen + STAGES * stage_bytes + 8 * STAGES);

  uint32_t ncols = 32;
  while (ncols < (uint32_t)a.bn) ncols <<= 1;

  if (warp == 0) {
    tmem_alloc(tmem_slot, ncols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bar_base + 8 * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_acc = *tmem_slot_ptr;

  const int nk = a.kpad / kChunkK;
  const uint32_t idesc = mma_idesc(a.bn, std::is_same<T, __nv_bfloat16>::value);
  bool ok = true;

  // prologue
#pragma unroll 1
  for (int c = 0; c < PF; ++c) {
    if (c < nk) gemm_load_chunk<T>(a, m0, n0, c, base + c * stage_bytes, base + c * stage_bytes + kTileABytes, tid);
    cp_async_commit();
  }

#pragma unroll 1
  for (int c = 0; c < nk; ++c) {
    const int s = c % STAGES;
    const int cn = c + PF;
    if (cn < nk) {
      const int sn = cn % STAGES;
      if (cn >= STAGES) {
        // stage sn last held chunk cn - STAGES; wait for its MMAs to finish
        if (!mbar_wait(bar_base + 8 * sn, (uint32_t)((cn / STAGES - 1) & 1))) ok = false;
      }
      gemm_load_chunk<T>(a, m0, n0, cn, base + sn * stage_bytes, base + sn * stage_bytes + kTileABytes, tid);
    }
    cp_async_commit();
    cp_async_wait<PF>();
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0 && ok) {
      tc_fence_after();
      const uint32_t sA = base + s * stage_bytes;
      const uint32_t sB = sA + kTileABytes;
#pragma unroll
      for (int kk = 0; kk < kChunkK / 16; ++kk) {
        tc_mma_f16(tmem_acc, sw128_desc(sA + kk * 32), sw128_desc(sB + kk * 32), idesc,
                   (c > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(bar_base + 8 * s);
    }
  }
  // all MMAs done <=> the last commit's barrier phase completed
  {
    const int cl = nk - 1;
    if (!mbar_wait(bar_base + 8 * (cl % STAGES), (uint32_t)((cl / STAGES) & 1))) ok = false;
  }
  cp_async_wait_all();
  tc_fence_after();
  const bool any_fail = __syncthreads_or(!ok);
  if (any_fail) {
    if (tid == 0 && a.err) atomicOr(a.err, 1);
  } else {
    // ------------------------------ epilogue ------------------------------
    const int r = warp * 32 + lane;
    const int m = m0 + r;
    const uint32_t trow = tmem_acc + ((uint32_t)(warp * 32) << 16);
    const bool valid = m < a.M;
    long long orow = m;
    if (valid && a.gidx) orow = __ldg(a.gidx + (long long)m * a.taps);
    const int fl = a.flags;
    float mk = 1.f;
    if (valid && (fl & (EPI_MASK | EPI_HEAD)) && a.rowmask) mk = __ldg(a.rowmask + orow);
    const int nch = a.bn / 16;

    float mean_a = 0.f, rstd_a = 1.f;
    if (fl & EPI_LN_A) {
      float cnt = 0.f, mean = 0.f, m2 = 0.f;
      for (int ch = 0; ch < nch; ++ch) {
        float v[16];
        tmem_ld16(trow + ch * 16, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] += __ldg(a.bias + n0 + ch * 16 + i);
        stats_merge(cnt, mean, m2, v);
      }
      mean_a = mean;
      rstd_a = rsqrtf(m2 / cnt + a.eps);
    }

    bool lnb_row = (fl & EPI_LN_B) != 0;
    if (lnb_row && (fl & EPI_LNB_TOKENS)) lnb_row = (orow % a.seq_len) < a.ntok;
    float cntb = 0.f, meanb = 0.f, m2b = 0.f;
    float head = 0.f;

    for (int ch = 0; ch < nch; ++ch) {
      const int c0 = n0 + ch * 16;
      float v[16];
      tmem_ld16(trow + ch * 16, v);
      if (!valid) continue;
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += __ldg(a.bias + c0 + i);
      if (fl & EPI_LN_A) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          v[i] = fmaf((v[i] - mean_a) * rstd_a, __ldg(a.ln_a_w + c0 + i), __ldg(a.ln_a_b + c0 + i));
      }
      if (fl & EPI_RELU) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = fmaxf(v[i], 0.f);
      }
      if (fl & EPI_GELU) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = gelu_erf(v[i]);
      }
      if (fl & EPI_HEAD) {
#pragma unroll
        for (int i = 0; i < 16; ++i) head = fmaf(fmaxf(v[i], 0.f), __ldg(a.head_w + c0 + i), head);
        continue;
      }
      if (fl & EPI_MASK) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] *= mk;
      }
      if (fl & EPI_RESID) {
        float x[16];
        load16_f32(a.out32 + orow * a.ld32 + c0, x);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = fmaf(v[i], __ldg(a.gamma + c0 + i), x[i]);
      }
      if (fl & EPI_POST_RELU) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = fmaxf(v[i], 0.f);
      }
      if (fl & EPI_RES16) {
        float x[16];
        load16<T>(a.res16, orow * a.ldr16 + c0, x);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = fmaxf(v[i] + x[i], 0.f);
      }
      if (fl & EPI_OUT32) store16_f32(a.out32 + orow * a.ld32 + c0, v);
      if (lnb_row) {
        stats_merge(cntb, meanb, m2b, v);
      } else if (fl & EPI_OUT16) {
        store16<T>(a.out16, orow * a.ld16 + c0, v);
      }
    }
    if (valid && (fl & EPI_HEAD) && a.head_out) a.head_out[m] = mk * (head + a.head_b);
    if (valid && lnb_row) {
      const float rstd_b = rsqrtf(m2b / cntb + a.eps);
      for (int ch = 0; ch < nch; ++ch) {
        const int c0 = n0 + ch * 16;
        float v[16];
        load16_f32(a.out32 + orow * a.ld32 + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          v[i] = fmaf((v[i] - meanb) * rstd_b, __ldg(a.ln_b_w + c0 + i), __ldg(a.ln_b_b + c0 + i));
        if (fl & EPI_OUT16) store16<T>(a.out16, orow * a.ld16 + c0, v);
        if (fl & EPI_OUT32B) store16_f32(a.out32b + orow * a.ld32b + c0, v);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_acc, ncols);
}

}  // namespace sb
