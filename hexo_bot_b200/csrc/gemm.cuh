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
//   warps 9-12 producers. When Cin is a multiple of 64, warp 9 alone feeds the
//              stage ring with TMA: 32 `tile::gather4` loads per 64-wide K
//              chunk pull the 128 gathered rows straight into the 128-byte
//              swizzled K-major layout (missing neighbours = out-of-range rows
//              -> zeros), one 2D TMA load brings the weight tile; both
//              complete on the stage's mbarrier. Otherwise all four warps
//              copy with cp.async and a software-pipelined proxy fence.
//   warp 8     issues tcgen05.mma (M=128, N=BN, K=16) from one thread into one
//              of two TMEM accumulators and commits each stage back to the
//              producers and each finished tile to the epilogue.
//   warps 0-7  epilogue, two warps per TMEM lane quadrant (one output row per
//              thread, one column half per warp); runs on accumulator j while
//              the MMA warp fills accumulator j^1.
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
  const float* head_b;     // [1] (EPI_HEAD)
  float* head_out;
  const int* skip_flag;    // if set and *skip_flag == skip_value the kernel returns at once
  int skip_value;          // (a device-side choice between two launched kernels)
  int seq_len;             // rows per position in the seq layout (for EPI_LNB_TOKENS)
  int ntok;
  int* err;                // device status word
  int tma_epi;             // epilogue stores / residual loads through TMA (set by the host)
  int orow_run;            // > 0 with orow_from_gidx: output rows run contiguously in blocks of this
                           // many GEMM rows (whole positions), so a 32-row quadrant starting at a
                           // multiple of 32 maps to 32 consecutive output rows
};

constexpr int kBlockM = 128;
constexpr int kChunkK = 64;        // 64 x 16-bit = one 128-byte swizzle row
constexpr int kTileABytes = kBlockM * 128;
// Warp roles: 0-7 epilogue (two per TMEM lane quadrant, one per column half),
// 8 MMA issue, 9-12 producers (TMA: warp 9 alone).
constexpr int kEpiWarps = 8;
constexpr int kMmaWarp = kEpiWarps;
constexpr int kProducerWarp0 = kMmaWarp + 1;
constexpr int kProducerWarps = 4;
constexpr int kGemmThreads = (kProducerWarp0 + kProducerWarps) * 32;  // 416
constexpr int kMaxTaps = 19;
constexpr int kMaxStages = 8;

__host__ __device__ constexpr int gemm_stage_bytes(int bn) { return kTileABytes + bn * 128; }
__host__ __device__ constexpr int gemm_gidx_bytes(int taps) { return 2 * kBlockM * taps * 4; }

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

// Chan's merge of a 16-value chunk into running (count, mean, M2). The
// chunk's sum and squared deviations are formed as balanced trees / four
// interleaved chains, so the dependent-add latency per chunk is ~6 operations
// instead of 16.
__device__ __forceinline__ void stats_merge(float& cnt, float& mean, float& m2, const float (&v)[16]) {
  float t[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) t[i] = v[2 * i] + v[2 * i + 1];
  const float s = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
  const float cm = s * (1.f / 16.f);
  float q[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float d = v[k] - cm;
    q[k] = d * d;
  }
#pragma unroll
  for (int i = 4; i < 16; ++i) {
    const float d = v[i] - cm;
    q[i & 3] = fmaf(d, d, q[i & 3]);
  }
  const float c2 = (q[0] + q[1]) + (q[2] + q[3]);
  const float tot = cnt + 16.f;
  const float delta = cm - mean;
  mean = fmaf(delta, 16.f / tot, mean);
  m2 += c2 + delta * delta * (cnt * 16.f / tot);
  cnt = tot;
}

// Exact (erf) GELU without erff: x * Phi(x) = max(x, 0) - |x| * (1 - Phi(|x|)),
// and 1 - Phi(u) = 0.5 * erfc(u / sqrt(2)) = exp(-u^2 / 2) * q(u) with q a
// degree-9 polynomial fit on u in [0, 4 sqrt(2)] (u clamped there; the term
// is below 1e-7 past it). tests/fit_gelu.py produces the coefficients and
// checks the error: at most ~7e-7 absolute against
// 0.5 * x * (1 + erf(x / sqrt(2))) over all float32 x. Straight-line code:
// 9 FMAs of Horner, one exp2 on the special-function unit, a NaN-propagating
// max (GELU(NaN) = NaN), no branch.
__device__ __forceinline__ float gelu_erf(float x) {
  const float u = fminf(fabsf(x), 5.656854249492380f);
  float p = -4.508463653e-06f;
  p = fmaf(p, u, 9.567350002e-05f);
  p = fmaf(p, u, -9.027047378e-04f);
  p = fmaf(p, u, 5.085092341e-03f);
  p = fmaf(p, u, -1.955406764e-02f);
  p = fmaf(p, u, 5.619602409e-02f);
  p = fmaf(p, u, -1.293920372e-01f);
  p = fmaf(p, u, 2.488136186e-01f);
  p = fmaf(p, u, -3.987478490e-01f);
  p = fmaf(p, u, 4.999889998e-01f);
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(u * (u * -0.72134752044448170f)));
  asm("max.NaN.f32 %0, %1, 0f00000000;" : "=f"(r) : "f"(x));
  return fmaf(-(u * p), e, r);
}

// ---- epilogue ---------------------------------------------------------------
// Eight warps: warp w reads TMEM lane quadrant w % 4 (32 accumulator rows, one
// row per thread) and column half w / 4 of the tile. Row-wise statistics
// (LayerNorm A / B, the policy-head dot product) are combined with the partner
// warp of the same quadrant through a small shared-memory exchange and a
// 64-thread named barrier. Values go from TMEM to registers 32 columns at a
// time and straight to / from global memory as 16-byte row pieces; every
// lane-dependent access is a single predicated instruction, so the warp stays
// converged for the .sync.aligned TMEM loads.

constexpr int kEpiVecFloats = 1024 + 6 * 256;   // bias (n_total) + six N-vectors
constexpr int kEpiXchBytes = 4 * 2 * 32 * 16;    // [quadrant][half][row] float4
constexpr int kEpiSmemBytes = kEpiVecFloats * 4 + kEpiXchBytes;

// TMA epilogue staging: kEpiWarps x (4 KB fp32 + 2 KB f16), 1024-aligned, plus
// one residual-load mbarrier per epilogue warp.
constexpr int kEpiTmaBytes = 8 * 6144;
__host__ __device__ constexpr int gemm_smem_bytes(int bn, int stages, int taps, bool tma_epi = false) {
  return 1024 + stages * gemm_stage_bytes(bn) + gemm_gidx_bytes(taps) + kEpiSmemBytes +
         (tma_epi ? (kEpiTmaBytes + 1024) : 0) + 8 * (2 * stages + 4 + 8) + 16;
}
// Stages that fit next to the gather-index double buffer and the epilogue data.
__host__ __device__ constexpr int gemm_stages(int bn, int taps, bool tma_epi = false) {
  int s = kMaxStages;
  while (s > 2 && gemm_smem_bytes(bn, s, taps, tma_epi) > 227 * 1024) --s;
  return s;
}

struct EpiVecs {
  const float* bias;  // [n_total]
  const float* lnaw;
  const float* lnab;
  const float* lnbw;
  const float* lnbb;
  const float* gamma;
  const float* headw;
};

// 32 TMEM columns (two x16 loads, one wait) of this thread's row.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr + 16));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// TMEM -> registers for `w` (16 or 32) columns starting at column c.
template <int W>
__device__ __forceinline__ void tmem_ldw(uint32_t taddr, float (&v)[32]) {
  if (W == 32) {
    tmem_ld32(taddr, v);
  } else {
    float t[16];
    tmem_ld16(taddr, t);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = t[i];
  }
}

template <int W>
__device__ __forceinline__ void ld_vec(const float* p, float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < W / 4; ++i) {
    const float4 f = reinterpret_cast<const float4*>(p)[i];
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}

template <int W>
__device__ __forceinline__ void stats_merge_w(float& cnt, float& mean, float& m2, const float (&v)[32]) {
  float a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = v[i];
  stats_merge(cnt, mean, m2, a);
  if (W == 32) {
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = v[16 + i];
    stats_merge(cnt, mean, m2, a);
  }
}

// Combine (cnt, mean, m2) with the partner warp's (Chan), always in the
// order (half 0, half 1) so both warps get bit-identical statistics.
__device__ __forceinline__ void stats_combine(float& cnt, float& mean, float& m2, float4* xme, const float4* xother,
                                              int bar_id, int half) {
  *xme = make_float4(cnt, mean, m2, 0.f);
  asm volatile("bar.sync %0, 64;\n" ::"r"(bar_id) : "memory");
  const float4 o = *xother;
  asm volatile("bar.sync %0, 64;\n" ::"r"(bar_id) : "memory");
  const float c0 = half ? o.x : cnt, u0 = half ? o.y : mean, q0 = half ? o.z : m2;
  const float c1 = half ? cnt : o.x, u1 = half ? mean : o.y, q1 = half ? m2 : o.z;
  const float tot = c0 + c1;
  const float delta = u1 - u0;
  const float w = tot > 0.f ? c1 / tot : 0.f;
  m2 = q0 + q1 + delta * delta * c0 * w;
  mean = fmaf(delta, w, u0);
  cnt = tot;
}

// fp32 row piece: 4 x 16-byte predicated stores / loads of W/4 ... columns.
template <int W>
__device__ __forceinline__ void st_row32(float* p, const float (&v)[32], bool ok) {
#pragma unroll
  for (int i = 0; i < W / 4; ++i)
    st_global_v4_if(p + 4 * i, make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]),
                                          __float_as_uint(v[4 * i + 2]), __float_as_uint(v[4 * i + 3])),
                    ok);
}
template <int W>
__device__ __forceinline__ void ld_row32(const float* p, float (&v)[32], bool ok) {
#pragma unroll
  for (int i = 0; i < W / 4; ++i) {
    const uint4 u = ld_global_v4_if(p + 4 * i, ok);
    v[4 * i] = __uint_as_float(u.x);
    v[4 * i + 1] = __uint_as_float(u.y);
    v[4 * i + 2] = __uint_as_float(u.z);
    v[4 * i + 3] = __uint_as_float(u.w);
  }
}
template <typename T, int W>
__device__ __forceinline__ void st_row16(void* p, const float (&v)[32], bool ok) {
#pragma unroll
  for (int i = 0; i < W / 8; ++i) {
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[8 * i + e]);
    st_global_v4_if(reinterpret_cast<T*>(p) + 8 * i, u, ok);
  }
}
template <typename T, int W>
__device__ __forceinline__ void ld_row16(const void* p, float (&v)[32], bool ok) {
#pragma unroll
  for (int i = 0; i < W / 8; ++i) {
    const uint4 u = ld_global_v4_if(reinterpret_cast<const T*>(p) + 8 * i, ok);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[8 * i + e] = to_f32<T>(h[e]);
  }
}

// Per-thread row context of one tile.
struct EpiRow {
  bool valid;       // GEMM row < M
  int mc;           // GEMM row, clamped to M - 1
  long long orow;   // output row
  float mk;         // row mask (EPI_MASK / EPI_HEAD)
  bool lnb_row;     // LayerNorm B applies to this row
};

// Row context of this thread for a tile (m_first: GEMM row of lane 0;
// tile_row: its row within the tile; rows at or past `tile_rows` within the
// tile, the padding of position-aligned tiles, or past M are never stored).
// Callers build it one tile ahead so the loads overlap the current tile.
__device__ __forceinline__ EpiRow make_epi_row(const GemmArgs& a, int m_first, int tile_row, int tile_rows,
                                               int lane) {
  // No branch depends on the lane: rows past M are clamped onto row M-1.
  EpiRow r;
  const int m = m_first + lane;
  r.valid = m < a.M && tile_row + lane < tile_rows;
  r.mc = r.valid ? m : a.M - 1;
  r.orow = (a.gidx && a.orow_from_gidx) ? (long long)__ldg(a.gidx + (long long)r.mc * a.taps) : (long long)r.mc;
  const int fl = a.flags;
  r.mk = ((fl & (EPI_MASK | EPI_HEAD)) && a.rowmask) ? __ldg(a.rowmask + r.orow) : 1.f;
  r.lnb_row = (fl & EPI_LN_B) != 0;
  if (fl & EPI_LNB_TOKENS) r.lnb_row = r.lnb_row && r.valid && (r.orow % a.seq_len) < a.ntok;
  return r;
}

// registers -> TMEM for W (16 or 32) columns of this thread's row
template <int W>
__device__ __forceinline__ void tmem_stw(uint32_t taddr, const float (&v)[32]) {
  uint32_t u[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(v[i]);
  if (W == 32) {
    tmem_st32(taddr, u);
  } else {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
        "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]),
        "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15])
        : "memory");
  }
}

// Main pass over one chunk of W columns [c, c + W) of the tile (tile-local
// column c, global column n0 + c).
// HEAVY: compiled with the residual / LayerNorm-B paths (flags EPI_RESID,
// EPI_RES16, EPI_LN_B); the light instantiation leaves them out so the other
// epilogues keep their registers.
template <typename T, int W, bool HEAVY>
__device__ __forceinline__ void epi_chunk_main(const GemmArgs& a, const EpiVecs& ev, const EpiRow& r, int n0, int c,
                                               uint32_t tcol, float mean_a, float rstd_a, float& head,
                                               float& cntb, float& meanb, float& m2b) {
  const int fl = HEAVY ? a.flags : (a.flags & ~(EPI_RESID | EPI_RES16 | EPI_LN_B));
  float v[32], t[32], x[32];
  // global loads first: their latency overlaps the TMEM read and the math
  if (HEAVY && (fl & EPI_RESID)) ld_row32<W>(a.out32 + r.orow * a.ld32 + n0 + c, x, r.valid);
  if (HEAVY && (fl & EPI_RES16))
    ld_row16<T, W>(reinterpret_cast<const T*>(a.res16) + r.orow * a.ldr16 + n0 + c, x, true);
  tmem_ldw<W>(tcol, v);
  ld_vec<W>(ev.bias + n0 + c, t);
#pragma unroll
  for (int i = 0; i < W; ++i) v[i] += t[i];
  if (fl & EPI_LN_A) {
    float w[32];
    ld_vec<W>(ev.lnaw + c, w);
    ld_vec<W>(ev.lnab + c, t);
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] = fmaf((v[i] - mean_a) * rstd_a, w[i], t[i]);
  }
  if (fl & EPI_RELU) {
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] = fmaxf(v[i], 0.f);
  }
  if (fl & EPI_GELU) {
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] = gelu_erf(v[i]);
  }
  if (fl & EPI_HEAD) {
    ld_vec<W>(ev.headw + c, t);
#pragma unroll
    for (int i = 0; i < W; ++i) head = fmaf(fmaxf(v[i], 0.f), t[i], head);
    return;
  }
  if (fl & EPI_MASK) {
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] *= r.mk;
  }
  if (fl & EPI_RESID) {
    ld_vec<W>(ev.gamma + c, t);
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] = fmaf(v[i], t[i], x[i]);
  }
  if (fl & EPI_POST_RELU) {
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] = fmaxf(v[i], 0.f);
  }
  if (fl & EPI_RES16) {
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] = fmaxf(v[i] + x[i], 0.f);
  }
  if (fl & EPI_LN_B) {
    stats_merge_w<W>(cntb, meanb, m2b, v);
    tmem_stw<W>(tcol, v);  // the accumulator columns hold v for the LayerNorm B pass
  }
  if (fl & (EPI_RESID | EPI_OUT32)) st_row32<W>(a.out32 + r.orow * a.ld32 + n0 + c, v, r.valid);
  if (fl & EPI_OUT16) st_row16<T, W>(reinterpret_cast<T*>(a.out16) + r.orow * a.ld16 + n0 + c, v,
                                     r.valid && !r.lnb_row);
}

// LayerNorm B over the row values the main pass parked in TMEM.
template <typename T, int W>
__device__ __forceinline__ void epi_chunk_lnb(const GemmArgs& a, const EpiVecs& ev, const EpiRow& r, int n0, int c,
                                              uint32_t tcol, float meanb, float rstd_b) {
  float v[32], w[32], t[32];
  tmem_ldw<W>(tcol, v);
  ld_vec<W>(ev.lnbw + c, w);
  ld_vec<W>(ev.lnbb + c, t);
#pragma unroll
  for (int i = 0; i < W; ++i) v[i] = fmaf((v[i] - meanb) * rstd_b, w[i], t[i]);
  const bool okb = r.valid && r.lnb_row;
  if (a.flags & EPI_OUT32B) st_row32<W>(a.out32b + r.orow * a.ld32b + n0 + c, v, okb);
  if (a.flags & EPI_OUT16) st_row16<T, W>(reinterpret_cast<T*>(a.out16) + r.orow * a.ld16 + n0 + c, v, okb);
}

template <typename T, bool HEAVY>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, const EpiVecs& ev, float4* xch, int bar_id,
                                              int half, const EpiRow& r, int n0, uint32_t tbase, int lane) {
  const int fl = HEAVY ? a.flags : (a.flags & ~(EPI_RESID | EPI_RES16 | EPI_LN_B));
  const int hw = a.bn >> 1;                     // columns per half
  const int c_lo = half * hw, c_hi = c_lo + hw;  // tile-local columns of this warp
  float4* xme = xch + half * 32 + lane;
  const float4* xot = xch + (half ^ 1) * 32 + lane;

  float mean_a = 0.f, rstd_a = 1.f;
  if (fl & EPI_LN_A) {
    float cnt = 0.f, mean = 0.f, m2 = 0.f;
    int c = c_lo;
    for (; c + 32 <= c_hi; c += 32) {
      float v[32], t[32];
      tmem_ldw<32>(tbase + c, v);
      ld_vec<32>(ev.bias + n0 + c, t);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += t[i];
      stats_merge_w<32>(cnt, mean, m2, v);
    }
    if (c < c_hi) {
      float v[32], t[32];
      tmem_ldw<16>(tbase + c, v);
      ld_vec<16>(ev.bias + n0 + c, t);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += t[i];
      stats_merge_w<16>(cnt, mean, m2, v);
    }
    stats_combine(cnt, mean, m2, xme, xot, bar_id, half);
    mean_a = mean;
    rstd_a = rsqrtf(m2 / cnt + a.eps);
  }

  float head = 0.f, cntb = 0.f, meanb = 0.f, m2b = 0.f;
  {
    int c = c_lo;
    for (; c + 32 <= c_hi; c += 32)
      epi_chunk_main<T, 32, HEAVY>(a, ev, r, n0, c, tbase + c, mean_a, rstd_a, head, cntb, meanb, m2b);
    if (c < c_hi) epi_chunk_main<T, 16, HEAVY>(a, ev, r, n0, c, tbase + c, mean_a, rstd_a, head, cntb, meanb, m2b);
  }

  if (fl & EPI_HEAD) {
    *xme = make_float4(head, 0.f, 0.f, 0.f);
    asm volatile("bar.sync %0, 64;\n" ::"r"(bar_id) : "memory");
    head = half ? xot->x + head : head + xot->x;
    asm volatile("bar.sync %0, 64;\n" ::"r"(bar_id) : "memory");
    if (a.head_out) st_global_f32_if(a.head_out + r.mc, r.mk * (head + __ldg(a.head_b)), r.valid && half == 0);
  }

  if (HEAVY && (fl & EPI_LN_B)) {
    stats_combine(cntb, meanb, m2b, xme, xot, bar_id, half);
    const float rstd_b = rsqrtf(m2b / fmaxf(cntb, 1.f) + a.eps);
    tmem_wait_st();  // the parked values are in TMEM before they are read back
    int c = c_lo;
    for (; c + 32 <= c_hi; c += 32) epi_chunk_lnb<T, 32>(a, ev, r, n0, c, tbase + c, meanb, rstd_b);
    if (c < c_hi) epi_chunk_lnb<T, 16>(a, ev, r, n0, c, tbase + c, meanb, rstd_b);
  }
}

// ---- TMA epilogue (identity-row GEMMs: output row = GEMM row) -------------------
// Each epilogue warp stages a 32-row x 32-column chunk of its rows in shared
// memory in the TMA's swizzled layout (fp32: 128-byte rows, 128B swizzle; f16:
// 64-byte rows, 64B swizzle) and one lane writes it with a bulk tensor store;
// the fp32 residual chunk arrives the same way (TMA load into the fp32
// staging, overwritten in place by the new values). Rows past the tensor are
// neither read nor written by the TMA unit.
constexpr int kEpiStageBytes = 4096 + 2048;  // per epilogue warp: fp32 chunk + f16 chunk

struct EpiTma {
  const CUtensorMap* o16;
  const CUtensorMap* o32;
  const CUtensorMap* o32b;
  uint8_t* st32;      // 4 KB, 1024-aligned
  uint8_t* st16;      // 2 KB, 1024-aligned
  uint32_t rbar;      // residual-load mbarrier of this warp
  int z;              // < 0: 2D maps (col, row); else 3D maps (col, row, z)
  const CUtensorMap* r16 = nullptr;  // 16-bit residual rows (EPI_RES16), staged through st16
};

__device__ __forceinline__ void tma_store_box(const EpiTma& e, const CUtensorMap* m, int col, int row, uint32_t src) {
  if (e.z < 0)
    tma_store_2d(m, col, row, src);
  else
    tma_store_3d(m, col, row, e.z, src);
}

__device__ __forceinline__ uint32_t st32_addr(int r, int i4) { return r * 128 + (((i4) ^ (r & 7)) << 4); }
__device__ __forceinline__ uint32_t st16_addr(int r, int i8) { return r * 64 + (((i8) ^ ((r >> 1) & 3)) << 4); }

__device__ __forceinline__ void stage_row32(uint8_t* st, int r, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
    *reinterpret_cast<float4*>(st + st32_addr(r, i)) = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
__device__ __forceinline__ void unstage_row32(const uint8_t* st, int r, float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = *reinterpret_cast<const float4*>(st + st32_addr(r, i));
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}
template <typename T>
__device__ __forceinline__ void unstage_row16(const uint8_t* st, int r, float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 u = *reinterpret_cast<const uint4*>(st + st16_addr(r, i));
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[8 * i + e] = to_f32<T>(h[e]);
  }
}
template <typename T>
__device__ __forceinline__ void stage_row16(uint8_t* st, int r, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[8 * i + e]);
    *reinterpret_cast<uint4*>(st + st16_addr(r, i)) = u;
  }
}

// Make this warp's staged rows visible to the TMA unit and store them.
__device__ __forceinline__ void stage_flush(const EpiTma& e, int lane, bool s32, const CUtensorMap* m32, bool s16,
                                            int col, int row) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (s32) tma_store_box(e, m32, col, row, smem_u32(e.st32));
    if (s16) tma_store_box(e, e.o16, col, row, smem_u32(e.st16));
    bulk_commit();
  }
}
// Before the staging is written again: the previous stores have read it.
__device__ __forceinline__ void stage_reuse(int lane) {
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
}

// Request the fp32 residual chunk [col, col + 32) x rows [m_first, +32) into
// the warp's fp32 staging once the stores that last read it are done
// (lane 0 issues; the caller's residual barrier phase is consumed by the
// matching wait in epilogue_tile_tma or epi_drain_resid).
__device__ __forceinline__ void epi_request_resid(const EpiTma& e, int col, int m_first, int lane) {
  if (lane == 0) {
    bulk_wait_read_all();
    mbar_arrive_expect_tx(e.rbar, 4096);
    if (e.z < 0)
      tma_load_2d(smem_u32(e.st32), e.o32, col, m_first, e.rbar);
    else
      tma_load_3d(smem_u32(e.st32), e.o32, col, m_first, e.z, e.rbar);
  }
  __syncwarp();
}
// Wait (bounded) for a requested residual chunk that no epilogue will read
// (the tile was abandoned after an error), so no copy lands later.
__device__ __forceinline__ void epi_drain_resid(const EpiTma& e, uint32_t& rphase) {
  mbar_wait(e.rbar, rphase);
  rphase ^= 1u;
}

// pre: the first residual chunk of this warp (columns [half * bn / 2, +32))
// was already requested with epi_request_resid. R16: the epilogue of the
// ray-tap conv, v = relu(acc + bias + res16) with the 16-bit residual rows
// staged through st16 (map e.r16).
template <typename T, bool HEAVY, bool R16 = false>
__device__ __forceinline__ void epilogue_tile_tma(const GemmArgs& a, const EpiVecs& ev, const EpiTma& e,
                                                  uint32_t& rphase, bool& ok, float4* xch, int bar_id, int half,
                                                  const EpiRow& r, int m_first, int n0, uint32_t tbase, int lane,
                                                  bool pre = false) {
  const int fl = R16 ? (a.flags & (EPI_RES16 | EPI_OUT16))
                     : HEAVY ? a.flags : (a.flags & ~(EPI_RESID | EPI_RES16 | EPI_LN_B));
  const int hw = a.bn >> 1;                     // columns per half (a multiple of 32 here)
  const int c_lo = half * hw, c_hi = c_lo + hw;
  float4* xme = xch + half * 32 + lane;
  const float4* xot = xch + (half ^ 1) * 32 + lane;

  float mean_a = 0.f, rstd_a = 1.f;
  if (fl & EPI_LN_A) {
    float cnt = 0.f, mean = 0.f, m2 = 0.f;
    for (int c = c_lo; c < c_hi; c += 32) {
      float v[32], t[32];
      tmem_ld32(tbase + c, v);
      ld_vec<32>(ev.bias + n0 + c, t);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += t[i];
      stats_merge_w<32>(cnt, mean, m2, v);
    }
    stats_combine(cnt, mean, m2, xme, xot, bar_id, half);
    mean_a = mean;
    rstd_a = rsqrtf(m2 / cnt + a.eps);
  }

  float cntb = 0.f, meanb = 0.f, m2b = 0.f;
  const bool lnb = HEAVY && (fl & EPI_LN_B);
  for (int c = c_lo; c < c_hi; c += 32) {
    float v[32], t[32], x[32];
    stage_reuse(lane);
    if (HEAVY && (fl & EPI_RESID)) {
      if (!(pre && c == c_lo)) epi_request_resid(e, n0 + c, m_first, lane);
      const bool got = ok && mbar_wait(e.rbar, rphase);
      ok = __all_sync(0xffffffffu, got) != 0;
      rphase ^= 1u;
      unstage_row32(e.st32, lane, x);
    }
    float x16[32];
    if (R16) {
      // the 16-bit residual chunk through the f16 staging (read back in place below)
      if (lane == 0) {
        mbar_arrive_expect_tx(e.rbar, 2048);
        if (e.z < 0)
          tma_load_2d(smem_u32(e.st16), e.r16, n0 + c, m_first, e.rbar);
        else
          tma_load_3d(smem_u32(e.st16), e.r16, n0 + c, m_first, e.z, e.rbar);
      }
      const bool got = ok && mbar_wait(e.rbar, rphase);
      ok = __all_sync(0xffffffffu, got) != 0;
      rphase ^= 1u;
      unstage_row16<T>(e.st16, lane, x16);
    }
    tmem_ld32(tbase + c, v);
    ld_vec<32>(ev.bias + n0 + c, t);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += t[i];
    if (fl & EPI_LN_A) {
      float w[32];
      ld_vec<32>(ev.lnaw + c, w);
      ld_vec<32>(ev.lnab + c, t);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaf((v[i] - mean_a) * rstd_a, w[i], t[i]);
    }
    if (fl & EPI_RELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
    }
    if (fl & EPI_GELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
    }
    if (fl & EPI_MASK) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= r.mk;
    }
    if (HEAVY && (fl & EPI_RESID)) {
      ld_vec<32>(ev.gamma + c, t);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaf(v[i], t[i], x[i]);
    }
    if (fl & EPI_POST_RELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
    }
    if (R16) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i] + x16[i], 0.f);
    }
    if (lnb) {
      stats_merge_w<32>(cntb, meanb, m2b, v);
      tmem_stw<32>(tbase + c, v);  // parked for the LayerNorm B pass
    }
    const bool s32 = (fl & (EPI_RESID | EPI_OUT32)) != 0;
    const bool s16 = (fl & EPI_OUT16) && !lnb;
    if (s32) stage_row32(e.st32, lane, v);
    if (s16) stage_row16<T>(e.st16, lane, v);
    if (s32 || s16) stage_flush(e, lane, s32, e.o32, s16, n0 + c, m_first);
  }

  if (lnb) {
    stats_combine(cntb, meanb, m2b, xme, xot, bar_id, half);
    const float rstd_b = rsqrtf(m2b / fmaxf(cntb, 1.f) + a.eps);
    tmem_wait_st();
    for (int c = c_lo; c < c_hi; c += 32) {
      float v[32], w[32], t[32];
      stage_reuse(lane);
      tmem_ld32(tbase + c, v);
      ld_vec<32>(ev.lnbw + c, w);
      ld_vec<32>(ev.lnbb + c, t);
      // rows outside LayerNorm B (non-token rows with EPI_LNB_TOKENS) keep v
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = r.lnb_row ? fmaf((v[i] - meanb) * rstd_b, w[i], t[i]) : v[i];
      const bool s32 = (fl & EPI_OUT32B) != 0;
      const bool s16 = (fl & EPI_OUT16) != 0;
      if (s32) stage_row32(e.st32, lane, v);
      if (s16) stage_row16<T>(e.st16, lane, v);
      if (s32 || s16) stage_flush(e, lane, s32, e.o32b, s16, n0 + c, m_first);
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

template <typename T, bool HEAVY, bool TMA_EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ws_kernel(const GemmArgs a, const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_o16,
                   const __grid_constant__ CUtensorMap tmap_o32, const __grid_constant__ CUtensorMap tmap_o32b,
                   int stages) {
  if (a.skip_flag) {
    pdl_wait();
    if (*reinterpret_cast<const volatile int*>(a.skip_flag) == a.skip_value) return;
  }
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
  float* vecs = reinterpret_cast<float*>(gbase + epi_off);             // epilogue vectors
  float4* xch_all = reinterpret_cast<float4*>(gbase + epi_off + kEpiVecFloats * 4);  // [4][2][32]
  // TMA epilogue staging, 1024-aligned (present when a.tma_epi)
  const uint32_t stg_off = (epi_off + kEpiSmemBytes + 1023u) & ~1023u;
  const uint32_t bar0 = base + (a.tma_epi ? stg_off + kEpiTmaBytes : epi_off + kEpiSmemBytes);
  const uint32_t full_bar = bar0;                 // [S]
  const uint32_t empty_bar = bar0 + 8 * S;        // [S]
  const uint32_t accf_bar = bar0 + 16 * S;        // [2]
  const uint32_t acce_bar = accf_bar + 16;        // [2]
  const uint32_t rload_bar = acce_bar + 16;       // [8] residual loads of the TMA epilogue
  const uint32_t tmem_slot = rload_bar + 64;
  volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const int acc_cols = (a.bn + 31) & ~31;
  uint32_t ncols = 32;
  while (ncols < (uint32_t)(2 * acc_cols)) ncols <<= 1;

  const int m_tiles = (a.M + kBlockM - 1) / kBlockM;
  const int n_tiles = a.n_total / a.bn;
  const int tiles = m_tiles * n_tiles;
  const int nk = a.kpad / kChunkK;
  const bool tma = a.use_tma != 0;

  pdl_launch_dependents();
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
    for (int i = 0; i < kEpiWarps; ++i) mbar_init(rload_bar + 8 * i, 1);
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
  // The epilogue reads and writes activations: it waits for the previous
  // kernel. The MMA issuer touches shared memory and TMEM only. The producer
  // waits before its first activation load (below).
  if (warp < kMmaWarp) pdl_wait();

  if (warp >= kProducerWarp0) {
    // ------------------------------------------------------------ producers
    const int pt = tid - kProducerWarp0 * 32;  // 0..127
    if (tma && warp != kProducerWarp0) {
      // only the first producer warp issues TMA
    } else {
      uint32_t it = 0;
      int j = 0;
      // The weights do not depend on the previous kernel: on the TMA path the
      // B tiles of the first ring stages go out before the wait.
      int pre = 0;
      if (tma && (int)blockIdx.x < tiles) {
        pre = S < nk ? S : nk;
        if (lane == 0) {
          const int n0 = (blockIdx.x % n_tiles) * a.bn;
          for (int c = 0; c < pre; ++c) {
            mbar_arrive_expect_tx(full_bar + 8 * c, kTileABytes + a.bn * 128);
            tma_load_2d(base + c * stage_bytes + kTileABytes, &tmap_b, c * kChunkK, n0, full_bar + 8 * c);
          }
        }
        __syncwarp();
      }
      pdl_wait();
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
            const bool b_sent = it < (uint32_t)pre;  // B tile already issued before the wait
            if (lane == 0 && !b_sent) mbar_arrive_expect_tx(full_bar + 8 * s, kTileABytes + a.bn * 128);
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
            if (lane == 0 && !b_sent) tma_load_2d(sB, &tmap_b, k0, n0, full_bar + 8 * s);
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
    const int quad = warp & 3;   // TMEM lanes [32 quad, 32 quad + 32)
    const int half = warp >> 2;  // column half of the tile
    const int bar_id = 3 + quad; // named barrier of the quadrant's warp pair
    float4* xch = xch_all + quad * 64;
    {
      float* bias_s = vecs;
      float* lnaw = vecs + 1024;
      const bool rowwise = a.bn == a.n_total;  // LN / head vectors only exist then
      for (int i = tid; i < a.n_total && i < 1024; i += kEpiWarps * 32) bias_s[i] = __ldg(a.bias + i);
      for (int i = tid; i < a.bn && rowwise; i += kEpiWarps * 32) {
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
    const EpiTma etma{&tmap_o16, &tmap_o32, &tmap_o32b, gbase + stg_off + warp * 6144,
                      gbase + stg_off + warp * 6144 + 4096, rload_bar + 8 * warp, -1};
    uint32_t rphase = 0;
    int j = 0;
    EpiRow row = make_epi_row(a, (blockIdx.x / n_tiles) * kBlockM + quad * 32, quad * 32, kBlockM, lane);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int nt = t % n_tiles;
      const int ab = j & 1;
      const int tn = t + gridDim.x;  // next tile's rows: loads in flight during this tile
      const EpiRow row_next = make_epi_row(a, (tn / n_tiles) * kBlockM + quad * 32, quad * 32, kBlockM, lane);
      // every lane waits (no lane-dependent control flow ahead of the
      // .sync.aligned TMEM loads of the epilogue)
      // this quadrant's first output row for the TMA epilogue: the GEMM row
      // itself, or (gathered rows in position blocks) its row in the output
      const int mq = (t / n_tiles) * kBlockM + quad * 32;
      const bool q_live = !a.gidx || mq < a.M;
      const int oq = (TMA_EPI && a.gidx && q_live) ? __ldg(a.gidx + (long long)mq * a.taps) : mq;
      // the residual rows of the first chunk are requested before the
      // accumulator is ready, so they arrive during the wait
      const bool pre = TMA_EPI && HEAVY && ok && q_live && (a.flags & EPI_RESID);
      if (pre) epi_request_resid(etma, nt * a.bn + half * (a.bn >> 1), oq, lane);
      const bool got = ok && mbar_wait_sleep(accf_bar + 8 * ab, (j >> 1) & 1);
      ok = __all_sync(0xffffffffu, got) != 0;
      // Both warps of a quadrant pair must agree on running the tile (they
      // exchange row statistics through named barriers): AND across the pair.
      ok = bar_red_and(bar_id, 64, ok);
      if (!ok && lane == 0 && a.err) atomicOr(a.err, SB_ERRBIT_EPILOGUE);
      tc_fence_after();
      if (!ok && pre) epi_drain_resid(etma, rphase);
      if (ok) {
        const uint32_t trow = tmem_base + ab * acc_cols + ((uint32_t)(quad * 32) << 16);
        if constexpr (TMA_EPI) {
          if (q_live)  // a gathered quadrant past M has no output rows
            epilogue_tile_tma<T, HEAVY>(a, ev, etma, rphase, ok, xch, bar_id, half, row, oq, nt * a.bn, trow, lane,
                                        pre);
        }
        else
          epilogue_tile<T, HEAVY>(a, ev, xch, bar_id, half, row, nt * a.bn, trow, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar + 8 * ab);
      row = row_next;
    }
    if (TMA_EPI && lane == 0) bulk_wait_all();  // the staging stays valid until the stores completed
    __syncwarp();
  }

  if (!ok && a.err) atomicOr(a.err, 1);
  cp_async_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem_base, ncols);
}

}  // namespace sb
