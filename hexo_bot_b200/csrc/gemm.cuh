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
// Persistent and warp-specialised: one CTA per SM walks 128-row x BN-column
// output tiles.
//   warps 0-3  producers. When Cin is a multiple of 64, warp 0 alone feeds the
//              stage ring with TMA: 32 `tile::gather4` loads per 64-wide K
//              chunk pull the 128 gathered rows straight into the 128-byte
//              swizzled K-major layout (missing neighbours = out-of-range rows
//              -> zeros), one 2D TMA load brings the weight tile; both
//              complete on the stage's mbarrier. Otherwise all four warps
//              copy with cp.async and a software-pipelined proxy fence.
//   warp 8     issues tcgen05.mma (M=128, N=BN, K=16) from one thread into one
//              of two TMEM accumulators and commits each stage back to the
//              producers and each finished tile to the epilogue.
//   warps 4-7  epilogue: one TMEM lane = one output row per thread, so the
//              LayerNorm statistics need no cross-thread reduction; runs on
//              accumulator j while the MMA warp fills accumulator j^1.
// Every mbarrier wait is bounded; a timeout sets a status bit and unwinds.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "ptx.cuh"

namespace sb {

// Status-word bits of a bounded wait that gave up, by the waiting role.
constexpr int SB_ERRBIT_PRODUCER = 1 << 4;   // stage never released by the MMA
constexpr int SB_ERRBIT_MMA_FULL = 1 << 5;   // stage never filled
constexpr int SB_ERRBIT_MMA_ACC = 1 << 6;    // accumulator never released by the epilogue
constexpr int SB_ERRBIT_EPILOGUE = 1 << 7;   // accumulator never committed

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
  long long a_rows;        // rows addressable in A
  int cin;                 // channels per tap (multiple of 8)
  int taps;                // T
  const int32_t* gidx;     // [M][T] source rows, -1 = zero; nullptr = identity (T == 1).
                           // The table must stay readable for 16 bytes past its end.
  int M;                   // output rows
  int orow_from_gidx;      // 1: GEMM row m is written to row gidx[m*T] (tap 0) of the outputs
                           // (seq layout); 0: to row m
  // B operand: [n_total][kpad] K-major 16-bit weights, kpad multiple of 64.
  const void* Bw;
  int kpad;
  int n_total;
  int bn;                  // N tile (multiple of 16, <= 256)
  int use_tma;             // producer path (set by the host)
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

constexpr int kBlockM = 128;
constexpr int kChunkK = 64;        // 64 x 16-bit = one 128-byte swizzle row
constexpr int kTileABytes = kBlockM * 128;
constexpr int kProducerWarps = 4;
constexpr int kEpiWarps = 4;
constexpr int kMmaWarp = kProducerWarps + kEpiWarps;
constexpr int kGemmThreads = (kMmaWarp + 1) * 32;  // 288
constexpr int kMaxTaps = 19;
constexpr int kMaxStages = 8;

__host__ __device__ constexpr int gemm_stage_bytes(int bn) { return kTileABytes + bn * 128; }
__host__ __device__ constexpr int gemm_gidx_bytes(int taps) { return 2 * kBlockM * taps * 4; }
__host__ __device__ constexpr int gemm_smem_bytes(int bn, int stages, int taps);

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

// ---- epilogue ---------------------------------------------------------------
// Each epilogue warp owns 32 accumulator rows (one TMEM lane per thread) and
// walks them in 32-column slabs: values are computed row-per-thread from TMEM
// and the shared-memory copies of the epilogue vectors, staged in swizzled
// shared memory, and moved to / from global memory with coalesced accesses
// (8 lanes per 128-byte fp32 row slab, 4 lanes per 64-byte 16-bit row slab).

constexpr int kSlab = 32;                       // columns per slab
constexpr int kStage32Bytes = 32 * kSlab * 4;   // 4 KB per warp
constexpr int kStage16Bytes = 32 * kSlab * 2;   // 2 KB per warp
constexpr int kEpiVecFloats = 1024 + 6 * 256;   // bias (n_total) + six N-vectors
constexpr int kEpiSmemBytes = kEpiWarps * (kStage32Bytes + kStage16Bytes) + kEpiVecFloats * 4;

__host__ __device__ constexpr int gemm_smem_bytes(int bn, int stages, int taps) {
  return 1024 + stages * gemm_stage_bytes(bn) + gemm_gidx_bytes(taps) + kEpiSmemBytes + 8 * (2 * stages + 4) + 16;
}
// Stages that fit next to the gather-index double buffer and epilogue staging.
__host__ __device__ constexpr int gemm_stages(int bn, int taps) {
  int s = kMaxStages;
  while (s > 2 && gemm_smem_bytes(bn, s, taps) > 227 * 1024) --s;
  return s;
}

struct EpiVecs {
  float* bias;  // [n_total]
  float* lnaw;
  float* lnab;
  float* lnbw;
  float* lnbb;
  float* gamma;
  float* headw;
};

// fp32 slab staging: row r, 16-byte piece p (4 floats) at r*128 + ((p ^ (r & 7)) << 4)
__device__ __forceinline__ uint32_t st32_off(int r, int p) { return r * 128 + ((p ^ (r & 7)) << 4); }
// 16-bit slab staging: row r, piece p (8 halves) at r*64 + ((p ^ ((r >> 1) & 3)) << 4)
__device__ __forceinline__ uint32_t st16_off(int r, int p) { return r * 64 + ((p ^ ((r >> 1) & 3)) << 4); }

// Coalesced copies of a 32-row x 32-float slab between global rows and the
// staging: 8 lanes per row, rows 4 i + lane / 8.
__device__ __forceinline__ void slab32_global_to_stage(uint8_t* st, const float* base, long long ld, int c0,
                                                       const long long (&rows)[8], const bool (&ok)[8], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3), p = lane & 7;
    *reinterpret_cast<uint4*>(st + st32_off(r, p)) = ld_global_v4_if(base + rows[i] * ld + c0 + 4 * p, ok[i]);
  }
}
__device__ __forceinline__ void slab32_stage_to_global(const uint8_t* st, float* base, long long ld, int c0,
                                                       const long long (&rows)[8], const bool (&ok)[8], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3), p = lane & 7;
    st_global_v4_if(base + rows[i] * ld + c0 + 4 * p, *reinterpret_cast<const uint4*>(st + st32_off(r, p)), ok[i]);
  }
}
template <typename T>
__device__ __forceinline__ void slab16_store(const float (&v)[kSlab], uint8_t* st16, void* out, long long ld,
                                             int c0, const long long (&r16)[4], const bool (&ok)[4], int lane) {
#pragma unroll
  for (int p = 0; p < kSlab / 8; ++p) {
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[8 * p + e]);
    *reinterpret_cast<uint4*>(st16 + st16_off(lane, p)) = u;
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 8 * i + (lane >> 2), p = lane & 3;
    st_global_v4_if(reinterpret_cast<T*>(out) + r16[i] * ld + c0 + 8 * p,
                    *reinterpret_cast<const uint4*>(st16 + st16_off(r, p)), ok[i]);
  }
  __syncwarp();
}

template <typename T>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, const EpiVecs& ev, uint8_t* st32, uint8_t* st16,
                                              int m_first, int n0, uint32_t tbase, int lane) {
  // No branch below depends on the lane: the tcgen05.ld / wait::ld of this
  // function are .sync.aligned and must run with the warp converged, so rows
  // past M are clamped onto row M-1 for every load and only the stores are
  // predicated.
  const int m = m_first + lane;
  const bool valid = m < a.M;
  const int mc = valid ? m : a.M - 1;
  const long long orow =
      (a.gidx && a.orow_from_gidx) ? (long long)__ldg(a.gidx + (long long)mc * a.taps) : (long long)mc;
  const int fl = a.flags;
  const float mk = ((fl & (EPI_MASK | EPI_HEAD)) && a.rowmask) ? __ldg(a.rowmask + orow) : 1.f;
  bool lnb_row = (fl & EPI_LN_B) != 0;
  if (fl & EPI_LNB_TOKENS) lnb_row = lnb_row && valid && (orow % a.seq_len) < a.ntok;

  long long r32[8];  // fp32 pattern rows 4 i + lane / 8
  bool ok32[8], okb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int src = 4 * i + (lane >> 3);
    // every lane executes every shuffle (no short-circuit around a
    // full-mask __shfl_sync: lanes that skipped it would leave the others
    // waiting forever)
    r32[i] = __shfl_sync(0xffffffffu, orow, src);
    ok32[i] = __shfl_sync(0xffffffffu, (int)valid, src) != 0;
    const bool lb = __shfl_sync(0xffffffffu, (int)lnb_row, src) != 0;
    okb[i] = ok32[i] && lb;
  }
  long long r16[4];  // 16-bit pattern rows 8 i + lane / 4
  bool raw16[4], lnb16[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int src = 8 * i + (lane >> 2);
    r16[i] = __shfl_sync(0xffffffffu, orow, src);
    const bool ok = __shfl_sync(0xffffffffu, (int)valid, src) != 0;
    const bool lb = __shfl_sync(0xffffffffu, (int)lnb_row, src) != 0;
    raw16[i] = ok && !lb;
    lnb16[i] = ok && lb;
  }

  const int nslab = a.bn / kSlab;
  float mean_a = 0.f, rstd_a = 1.f;
  if (fl & EPI_LN_A) {
    float cnt = 0.f, mean = 0.f, m2 = 0.f;
    for (int ch = 0; ch < a.bn / 16; ++ch) {
      float v[16];
      tmem_ld16(tbase + ch * 16, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += ev.bias[n0 + ch * 16 + i];
      stats_merge(cnt, mean, m2, v);
    }
    mean_a = mean;
    rstd_a = rsqrtf(m2 / cnt + a.eps);
  }

  float cntb = 0.f, meanb = 0.f, m2b = 0.f;
  float head = 0.f;
  const bool need32 = (fl & (EPI_RESID | EPI_OUT32)) != 0;
  for (int sl = 0; sl < nslab; ++sl) {
    const int c0 = sl * kSlab;
    if (fl & EPI_RESID) {
      slab32_global_to_stage(st32, a.out32, a.ld32, n0 + c0, r32, ok32, lane);
      __syncwarp();
    }
    float lo[16], hi[16];
    tmem_ld16(tbase + c0, lo);
    tmem_ld16(tbase + c0 + 16, hi);
    float v[kSlab];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = lo[i];
      v[16 + i] = hi[i];
    }
#pragma unroll
    for (int i = 0; i < kSlab; ++i) {
      float x = v[i] + ev.bias[n0 + c0 + i];
      if (fl & EPI_LN_A) x = fmaf((x - mean_a) * rstd_a, ev.lnaw[c0 + i], ev.lnab[c0 + i]);
      if (fl & EPI_RELU) x = fmaxf(x, 0.f);
      if (fl & EPI_GELU) x = gelu_erf(x);
      v[i] = x;
    }
    if (fl & EPI_HEAD) {
#pragma unroll
      for (int i = 0; i < kSlab; ++i) head = fmaf(fmaxf(v[i], 0.f), ev.headw[c0 + i], head);
      continue;
    }
#pragma unroll
    for (int i = 0; i < kSlab; ++i) {
      float x = v[i];
      if (fl & EPI_MASK) x *= mk;
      if (fl & EPI_RESID) {
        const float xr = reinterpret_cast<const float*>(st32 + st32_off(lane, i >> 2))[i & 3];
        x = fmaf(x, ev.gamma[c0 + i], xr);
      }
      if (fl & EPI_POST_RELU) x = fmaxf(x, 0.f);
      v[i] = x;
    }
    if (fl & EPI_RES16) {
      float q0[16], q1[16];
      load16<T>(a.res16, orow * a.ldr16 + n0 + c0, q0);
      load16<T>(a.res16, orow * a.ldr16 + n0 + c0 + 16, q1);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = fmaxf(v[i] + q0[i], 0.f);
        v[16 + i] = fmaxf(v[16 + i] + q1[i], 0.f);
      }
    }
    if (fl & EPI_LN_B) {  // statistics on every lane (uniform branch); used where lnb_row
      float s0[16], s1[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        s0[i] = v[i];
        s1[i] = v[16 + i];
      }
      stats_merge(cntb, meanb, m2b, s0);
      stats_merge(cntb, meanb, m2b, s1);
    }
    if (need32) {
      __syncwarp();
#pragma unroll
      for (int p = 0; p < kSlab / 4; ++p)
        *reinterpret_cast<float4*>(st32 + st32_off(lane, p)) =
            make_float4(v[4 * p], v[4 * p + 1], v[4 * p + 2], v[4 * p + 3]);
      __syncwarp();
      slab32_stage_to_global(st32, a.out32, a.ld32, n0 + c0, r32, ok32, lane);
      __syncwarp();
    }
    if (fl & EPI_OUT16) slab16_store<T>(v, st16, a.out16, a.ld16, n0 + c0, r16, raw16, lane);
  }
  if ((fl & EPI_HEAD) && a.head_out) st_global_f32_if(a.head_out + mc, mk * (head + a.head_b), valid);

  // pass 3: LayerNorm_b of the stored fp32 rows (re-read through the staging)
  if ((fl & EPI_LN_B) && __any_sync(0xffffffffu, lnb_row)) {
    const float rstd_b = lnb_row ? rsqrtf(m2b / cntb + a.eps) : 1.f;
    for (int sl = 0; sl < nslab; ++sl) {
      const int c0 = sl * kSlab;
      slab32_global_to_stage(st32, a.out32, a.ld32, n0 + c0, r32, ok32, lane);
      __syncwarp();
      float v[kSlab];
#pragma unroll
      for (int i = 0; i < kSlab; ++i) {
        const float x = reinterpret_cast<const float*>(st32 + st32_off(lane, i >> 2))[i & 3];
        v[i] = fmaf((x - meanb) * rstd_b, ev.lnbw[c0 + i], ev.lnbb[c0 + i]);
      }
      __syncwarp();
      if (fl & EPI_OUT32B) {
#pragma unroll
        for (int p = 0; p < kSlab / 4; ++p)
          *reinterpret_cast<float4*>(st32 + st32_off(lane, p)) =
              make_float4(v[4 * p], v[4 * p + 1], v[4 * p + 2], v[4 * p + 3]);
        __syncwarp();
        slab32_stage_to_global(st32, a.out32b, a.ld32b, n0 + c0, r32, okb, lane);
        __syncwarp();
      }
      if (fl & EPI_OUT16) slab16_store<T>(v, st16, a.out16, a.ld16, n0 + c0, r16, lnb16, lane);
    }
  }
}

// cp.async producer for one K chunk (used when Cin is not a multiple of 64):
// thread `pt` of the 128 producer threads copies 16-byte pieces of 8 A rows
// and BN/16 B rows into the 128-byte-swizzled stage.
template <typename T>
__device__ __forceinline__ void cpasync_chunk(const GemmArgs& a, const int32_t* gs, int m0, int n0, int chunk,
                                              uint32_t sA, uint32_t sB, int pt) {
  const int kbase = chunk * kChunkK;
  const int p = pt & 7;
  const int rsub = pt >> 3;
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
    if (m < a.M && k < ktot) src_row = a.gidx ? (long long)gs[r * a.taps + tap] : m;
    const void* src = X;
    uint32_t bytes = 0;
    if (src_row >= 0 && src_row < a.a_rows) {
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

template <typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ws_kernel(const GemmArgs a, const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, int stages) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = stages;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t stage_bytes = gemm_stage_bytes(a.bn);
  const uint32_t gidx_off = S * stage_bytes;
  int32_t* gsm = reinterpret_cast<int32_t*>(gbase + gidx_off);        // [2][128 * taps]
  const uint32_t epi_off = gidx_off + gemm_gidx_bytes(a.taps);
  uint8_t* epi_smem = gbase + epi_off;                                 // staging + vectors
  const uint32_t bar0 = base + epi_off + kEpiSmemBytes;
  const uint32_t full_bar = bar0;                 // [S]
  const uint32_t empty_bar = bar0 + 8 * S;        // [S]
  const uint32_t accf_bar = bar0 + 16 * S;        // [2]
  const uint32_t acce_bar = accf_bar + 16;        // [2]
  const uint32_t tmem_slot = acce_bar + 16;
  volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const int acc_cols = (a.bn + 31) & ~31;
  uint32_t ncols = 32;
  while (ncols < (uint32_t)(2 * acc_cols)) ncols <<= 1;

  const int m_tiles = (a.M + kBlockM - 1) / kBlockM;
  const int n_tiles = a.n_total / a.bn;
  const int tiles = m_tiles * n_tiles;
  const int nk = a.kpad / kChunkK;
  const bool tma = a.use_tma != 0;

  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, ncols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar + 8 * s, tma ? 1 : kProducerWarps * 32);
      mbar_init(empty_bar + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf_bar + 8 * i, 1);
      mbar_init(acce_bar + 8 * i, kEpiWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    if (tma) {
      prefetch_tmap(&tmap_a);
      prefetch_tmap(&tmap_b);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;
  bool ok = true;

  if (warp < kProducerWarps) {
    // ------------------------------------------------------------ producers
    const int pt = tid;  // 0..127
    if (tma && warp != 0) {
      // only warp 0 issues TMA
    } else {
      uint32_t it = 0;
      int j = 0;
      const int gwords = kBlockM * a.taps;
      // stage the gather rows of tile t into gather buffer `buf` (cp.async)
      auto fetch_gidx = [&](int t, int buf) {
        const int mt = t / n_tiles;
        const long long first = (long long)mt * kBlockM * a.taps;          // word offset
        const long long total = (long long)a.M * a.taps;
        const uint32_t dst = smem_u32(gsm + buf * gwords);
        const int nthreads = tma ? 32 : kProducerWarps * 32;
        // Whole 16-byte pieces only: gather tables carry >= 16 bytes of
        // readable slack past M * taps words (rows >= M are never used).
        for (int q = pt; q * 4 < gwords; q += nthreads) {
          const long long w = first + q * 4;
          const bool in = w < total;
          cp_async16(dst + q * 16, in ? (const void*)(a.gidx + w) : (const void*)a.gidx, in ? 16u : 0u);
        }
        cp_async_commit();
      };
      int t = blockIdx.x;
      if (a.gidx && t < tiles) fetch_gidx(t, 0);
      constexpr int kLag = 2;  // cp.async path: chunks in flight before signalling (< stages)
      for (; t < tiles; t += gridDim.x, ++j) {
        const int nt = t % n_tiles, mt = t / n_tiles;
        const int m0 = mt * kBlockM, n0 = nt * a.bn;
        const int32_t* gs = gsm + (j & 1) * gwords;
        if (a.gidx) {
          if (tma) {
            cp_async_wait_all();
            __syncwarp();
          } else {
            cp_async_wait_all();
            asm volatile("bar.sync 1, 128;\n" ::: "memory");
          }
          if (t + (int)gridDim.x < tiles) fetch_gidx(t + gridDim.x, (j + 1) & 1);
        }
        for (int c = 0; c < nk; ++c, ++it) {
          const int s = it % S;
          if (lane == 0 && ok && !mbar_wait_sleep(empty_bar + 8 * s, ((it / S) & 1) ^ 1)) {
            ok = false;
            if (a.err) atomicOr(a.err, SB_ERRBIT_PRODUCER);
          }
          __syncwarp();
          const uint32_t sA = base + s * stage_bytes;
          const uint32_t sB = sA + kTileABytes;
          if (tma) {
            const int k0 = c * kChunkK;
            const int tap = k0 / a.cin;
            const int col = k0 - tap * a.cin;
            if (lane == 0) mbar_arrive_expect_tx(full_bar + 8 * s, kTileABytes + a.bn * 128);
            __syncwarp();
            if (a.gidx) {
              int rr[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int r = lane * 4 + i;
                rr[i] = m0 + r < a.M ? gs[r * a.taps + tap] : -1;
              }
              tma_gather4(sA + lane * 512, &tmap_a, col, rr[0], rr[1], rr[2], rr[3], full_bar + 8 * s);
            } else if (lane == 0) {
              // contiguous rows: one 128-row box (rows past the end read as zeros)
              tma_load_2d(sA, &tmap_a, col, m0, full_bar + 8 * s);
            }
            if (lane == 0) tma_load_2d(sB, &tmap_b, k0, n0, full_bar + 8 * s);
          } else {
            cpasync_chunk<T>(a, gs, m0, n0, c, sA, sB, pt);
            cp_async_commit();
            // Signal chunk it - kLag once this thread's copies for it have
            // landed: the two newer groups may still be in flight.
            if (it >= (uint32_t)kLag) {
              cp_async_wait<kLag>();
              fence_proxy_async_smem();
              mbar_arrive(full_bar + 8 * ((it - kLag) % S));
            }
          }
        }
      }
      if (!tma) {
        cp_async_wait_all();
        fence_proxy_async_smem();
        for (uint32_t q = it >= (uint32_t)kLag ? it - kLag : 0; q < it; ++q) mbar_arrive(full_bar + 8 * (q % S));
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t idesc = mma_idesc(a.bn, std::is_same<T, __nv_bfloat16>::value);
      // Descriptors of stage 0; stage s adds s * stage_bytes / 16 to the
      // start-address field and each 16-wide K step adds 32 B (2 units).
      const uint64_t adesc0 = sw128_desc(base);
      const uint64_t bdesc0 = sw128_desc(base + kTileABytes);
      const uint64_t stage_step = stage_bytes >> 4;
      uint32_t it = 0, s = 0, ph = 0;
      int j = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
        const int ab = j & 1;
        if (ok && !mbar_wait(acce_bar + 8 * ab, ((j >> 1) & 1) ^ 1)) {
          ok = false;
          if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_ACC);
        }
        tc_fence_after();
        const uint32_t dacc = tmem_base + ab * acc_cols;
        for (int c = 0; c < nk; ++c, ++it) {
          if (ok && !mbar_wait(full_bar + 8 * s, ph)) {
            ok = false;
            if (a.err) atomicOr(a.err, SB_ERRBIT_MMA_FULL);
          }
          tc_fence_after();
          const uint64_t ad = adesc0 + s * stage_step;
          const uint64_t bd = bdesc0 + s * stage_step;
          if (ok) {
            tc_mma_f16(dacc, ad, bd, idesc, c > 0 ? 1u : 0u);
            tc_mma_f16_acc(dacc, ad + 2, bd + 2, idesc);
            tc_mma_f16_acc(dacc, ad + 4, bd + 4, idesc);
            tc_mma_f16_acc(dacc, ad + 6, bd + 6, idesc);
          }
          tc_commit(empty_bar + 8 * s);
          if (++s == (uint32_t)S) {
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
    const int ew = warp - kProducerWarps;  // == warp % 4: TMEM lanes [32 ew, 32 ew + 32)
    uint8_t* st32 = epi_smem + ew * (kStage32Bytes + kStage16Bytes);
    uint8_t* st16 = st32 + kStage32Bytes;
    float* vecs = reinterpret_cast<float*>(epi_smem + kEpiWarps * (kStage32Bytes + kStage16Bytes));
    EpiVecs ev{vecs, vecs + 1024, vecs + 1024 + 256, vecs + 1024 + 512, vecs + 1024 + 768, vecs + 1024 + 1024,
               vecs + 1024 + 1280};
    {
      const int et = tid - kProducerWarps * 32;  // 0..127
      const bool rowwise = a.bn == a.n_total;    // LN / head vectors only exist then
      for (int i = et; i < a.n_total && i < 1024; i += kEpiWarps * 32) ev.bias[i] = __ldg(a.bias + i);
      for (int i = et; i < a.bn && rowwise; i += kEpiWarps * 32) {
        ev.lnaw[i] = a.ln_a_w ? __ldg(a.ln_a_w + i) : 0.f;
        ev.lnab[i] = a.ln_a_b ? __ldg(a.ln_a_b + i) : 0.f;
        ev.lnbw[i] = a.ln_b_w ? __ldg(a.ln_b_w + i) : 0.f;
        ev.lnbb[i] = a.ln_b_b ? __ldg(a.ln_b_b + i) : 0.f;
        ev.headw[i] = a.head_w ? __ldg(a.head_w + i) : 0.f;
        ev.gamma[i] = a.gamma ? __ldg(a.gamma + i) : 0.f;
      }
      asm volatile("bar.sync 2, 128;\n" ::: "memory");
    }
    int j = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int nt = t % n_tiles, mt = t / n_tiles;
      const int ab = j & 1;
      // every lane waits (no lane-dependent control flow ahead of the
      // .sync.aligned TMEM loads of the epilogue)
      const bool got = ok && mbar_wait_sleep(accf_bar + 8 * ab, (j >> 1) & 1);
      ok = __all_sync(0xffffffffu, got) != 0;
      if (!ok && lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_EPILOGUE);
      tc_fence_after();
      if (ok) {
        const uint32_t trow = tmem_base + ab * acc_cols + ((uint32_t)(ew * 32) << 16);
        epilogue_tile<T>(a, ev, st32, st16, mt * kBlockM + ew * 32, nt * a.bn, trow, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar + 8 * ab);
    }
  }

  if (!ok && a.err) atomicOr(a.err, 1);
  cp_async_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem_base, ncols);
}

}  // namespace sb
