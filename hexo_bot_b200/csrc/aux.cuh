// Small memory-bound kernels around the tensor-core layers: input staging and
// index tables, token rows, the value / moves-left heads with their binned
// decode, the legal-prefix prior softmax, and weight packing.
#pragma once

#include "ptx.cuh"

namespace sb {

constexpr int kNumTok = 8;
constexpr int kNumFeat = 15;
constexpr int kFeatPad = 16;
constexpr int kBins = 65;

template <typename I>
__device__ __forceinline__ long long load_int(const void* p, long long i) {
  return (long long)reinterpret_cast<const I*>(p)[i];
}

__device__ __forceinline__ long long load_index(const void* p, int dtype, long long i) {
  switch (dtype) {
    case 3: return load_int<long long>(p, i);
    case 4: return load_int<int32_t>(p, i);
    case 6: return load_int<int16_t>(p, i);
    case 7: {
      const long long v = load_int<uint16_t>(p, i);
      return v == 0xFFFF ? -1 : v;
    }
    case 5: return load_int<uint8_t>(p, i);
    default: return 0;
  }
}

__device__ __forceinline__ float load_float(const void* p, int dtype, long long i) {
  switch (dtype) {
    case 0: return reinterpret_cast<const float*>(p)[i];
    case 1: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case 2: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    default: return 0.f;
  }
}

__device__ __forceinline__ float load_mask(const void* p, int dtype, long long i) {
  if (dtype == 0) return reinterpret_cast<const float*>(p)[i] != 0.f ? 1.f : 0.f;
  return reinterpret_cast<const uint8_t*>(p)[i] != 0 ? 1.f : 0.f;
}

struct PrepArgs {
  const void* feats; int feats_dtype;
  const void* nbr; int nbr_dtype;
  const void* mask; int mask_dtype;
  const void* coords; int coords_dtype;
  int B, npad, S;
  __half* feat16;     // (B*S, 16)
  int32_t* gidx;      // (B*npad, 7) absolute seq rows, -1 = missing
  float* rowmask;     // (B*S)
  int32_t* coords32;  // (B*npad, 2)
  int* grid_flag;     // set to 1 here (grid_geom_kernel clears it), or NULL
  int* err;
};

// Inputs of one group of rows of the serve payload (the evaluator's wire ABI,
// shrimp-rs payload.rs:108-158): CSR over support nodes, rows [row0, row0 + B)
// padded to npad cells each.
struct PrepCsrArgs {
  const void* feats; int feats_dtype;  // (total_nodes, 15)
  const int16_t* qr;                   // (total_nodes, 2) hex coordinates
  const uint16_t* nbr;                 // (total_nodes, 6) row-local neighbours, 0xFFFF = missing
  const int64_t* offsets;              // (rows + 1) first node of each payload row
  int row0;
  int B, npad, S;
  __half* feat16;
  int32_t* gidx;
  float* rowmask;
  int32_t* coords32;
  int32_t* seq_lens;  // (B) 8 tokens + the row's node count: rows past it are padding
  int* err;
};

// One thread per cell: stage features (f16, padded to 16 channels), the
// absolute-row gather table (tap 0 = self, taps 1..6 = DIRECTIONS neighbours;
// reference trunk gather_idx, model.py:860-863), the row mask and int32 coords.
__global__ void prep_cells_kernel(const PrepArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i == 0 && a.grid_flag) *a.grid_flag = 1;
  const long long ncell = (long long)a.B * a.npad;
  if (i < ncell) {
    const int b = (int)(i / a.npad);
    const int n = (int)(i - (long long)b * a.npad);
    const long long row = (long long)b * a.S + kNumTok + n;
    __align__(16) __half f[kFeatPad];
#pragma unroll
    for (int c = 0; c < kNumFeat; ++c) f[c] = __float2half_rn(load_float(a.feats, a.feats_dtype, i * kNumFeat + c));
    f[kNumFeat] = __float2half_rn(0.f);
    uint4* dst = reinterpret_cast<uint4*>(a.feat16 + row * kFeatPad);
    dst[0] = reinterpret_cast<const uint4*>(f)[0];
    dst[1] = reinterpret_cast<const uint4*>(f)[1];
    int32_t* g = a.gidx + i * 7;
    g[0] = (int32_t)row;
    for (int k = 0; k < 6; ++k) {
      const long long v = load_index(a.nbr, a.nbr_dtype, i * 6 + k);
      int32_t out = -1;
      if (v >= 0 && v < a.npad) {
        out = (int32_t)((long long)b * a.S + kNumTok + v);
      } else if (v > a.npad && a.err) {
        atomicOr(a.err, 2);
      }
      g[1 + k] = out;
    }
    a.rowmask[row] = load_mask(a.mask, a.mask_dtype, i);
    a.coords32[2 * i] = (int32_t)load_index(a.coords, a.coords_dtype, 2 * i);
    a.coords32[2 * i + 1] = (int32_t)load_index(a.coords, a.coords_dtype, 2 * i + 1);
  }
  // token rows of the row mask
  if (i < (long long)a.B * kNumTok) {
    const long long b = i / kNumTok, t = i - b * kNumTok;
    a.rowmask[b * a.S + t] = 1.f;
  }
}

// prep_cells_kernel for one group of payload rows: node n of row b is cell n
// of position b (the support order [legal | stones | halo] is kept), cells past
// the row's node count are padding (zero features, no neighbours, mask 0,
// coordinates 0: the reference evaluator's per-group pack, inference.py:865-897).
__global__ void prep_csr_kernel(const PrepCsrArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long ncell = (long long)a.B * a.npad;
  if (i < ncell) {
    const int b = (int)(i / a.npad);
    const int n = (int)(i - (long long)b * a.npad);
    const long long o0 = __ldg(a.offsets + a.row0 + b);
    const long long size = __ldg(a.offsets + a.row0 + b + 1) - o0;
    const long long row = (long long)b * a.S + kNumTok + n;
    const bool real = n < size;
    const long long node = o0 + n;
    __align__(16) __half f[kFeatPad];
#pragma unroll
    for (int c = 0; c < kNumFeat; ++c)
      f[c] = __float2half_rn(real ? load_float(a.feats, a.feats_dtype, node * kNumFeat + c) : 0.f);
    f[kNumFeat] = __float2half_rn(0.f);
    uint4* dst = reinterpret_cast<uint4*>(a.feat16 + row * kFeatPad);
    dst[0] = reinterpret_cast<const uint4*>(f)[0];
    dst[1] = reinterpret_cast<const uint4*>(f)[1];
    int32_t* g = a.gidx + i * 7;
    g[0] = (int32_t)row;
    for (int k = 0; k < 6; ++k) {
      int32_t out = -1;
      if (real) {
        const int v = __ldg(a.nbr + node * 6 + k);
        if (v < size && v < a.npad) {
          out = (int32_t)((long long)b * a.S + kNumTok + v);
        } else if (v != 0xFFFF && a.err) {
          atomicOr(a.err, 2);
        }
      }
      g[1 + k] = out;
    }
    a.rowmask[row] = real ? 1.f : 0.f;
    a.coords32[2 * i] = real ? (int32_t)__ldg(a.qr + 2 * node) : 0;
    a.coords32[2 * i + 1] = real ? (int32_t)__ldg(a.qr + 2 * node + 1) : 0;
    if (n == 0) {
      if (size > a.npad && a.err) atomicOr(a.err, 4);
      a.seq_lens[b] = kNumTok + (int)min(size, (long long)a.npad);
    }
  }
  if (i < (long long)a.B * kNumTok) {
    const long long b = i / kNumTok, t = i - b * kNumTok;
    a.rowmask[b * a.S + t] = 1.f;
  }
}

// Token rows of the residual stream (learned tokens) and of the first
// attention block's LN1 input (precomputed per weights).
__global__ void init_tokens_kernel(const float* tokens, const __half* tokens_ln16, int B, int S, int C,
                                   float* seq32, __half* xa16) {
  pdl_launch_dependents();
  pdl_wait();
  // one thread per 4 consecutive channels of one token row (C is a multiple of 32)
  const int per4 = kNumTok * C / 4;  // quads per position
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= B * per4) return;
  const int b = q / per4;
  const int r = (q - b * per4) * 4;  // value index within the position's token block
  const long long o = ((long long)b * S + r / C) * C + r % C;
  *reinterpret_cast<float4*>(seq32 + o) = __ldg(reinterpret_cast<const float4*>(tokens + r));
  *reinterpret_cast<uint2*>(xa16 + o) = __ldg(reinterpret_cast<const uint2*>(tokens_ln16 + r));
}

// gather_idx in the reference's row-local convention (missing -> Npad).
__global__ void gather_index_kernel(const void* nbr, int dtype, int B, int npad, int32_t* out, int* err) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * npad) return;
  const int n = (int)(i % npad);
  out[i * 7] = n;
  for (int k = 0; k < 6; ++k) {
    const long long v = load_index(nbr, dtype, i * 6 + k);
    int32_t o = npad;
    if (v >= 0 && v < npad) o = (int32_t)v;
    else if (v > npad && err) atomicOr(err, 2);
    out[i * 7 + 1 + k] = o;
  }
}

// Row-local gather table -> absolute rows of a (B, npad, C) tensor.
__global__ void absolute_gidx_kernel(const int32_t* local, int B, int npad, int taps, int32_t* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * npad * taps) return;
  const long long row = i / taps;
  const long long b = row / npad;
  const int v = local[i];
  out[i] = (v >= 0 && v < npad) ? (int32_t)(b * npad + v) : -1;
}

// Per-position shared neighbour table (N, T) -> absolute rows for B positions.
__global__ void shared_gidx_kernel(const int32_t* nbr, int B, int n, int taps, int32_t* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * n * taps) return;
  const long long b = i / ((long long)n * taps);
  const int j = (int)(i - b * n * taps);
  const int v = nbr[j];
  out[i] = (v >= 0 && v < n) ? (int32_t)(b * n + v) : -1;
}

__global__ void mask_to_float_kernel(const uint8_t* m, long long n, float* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = m[i] ? 1.f : 0.f;
}

// Bias row of one (query, key) pair of the joint sequence (model.py:677-716):
// token/token 236, token->cell 235, cell->token 234, cell/cell = LUT of the
// clamped (key - query) offset.
__device__ __forceinline__ int pair_row(int qi, int ki, int qq, int qr, int kq, int kr, const uint8_t* lut) {
  const bool qt = qi < kNumTok, kt = ki < kNumTok;
  if (qt) return kt ? 236 : 235;
  if (kt) return 234;
  const int dq = min(max(kq - qq, -17), 17);
  const int dr = min(max(kr - qr, -17), 17);
  return lut[(dq + 17) * 35 + dr + 17];
}

// (B, S, S) uint8 pair table; dead cell keys -> 237 (model.py:762-792).
__global__ void pair_u8_kernel(const void* coords, int cdtype, const void* mask, int mdtype, int B, int npad,
                               const uint8_t* lut, uint8_t* out) {
  const int S = npad + kNumTok;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * S * S) return;
  const long long b = i / ((long long)S * S);
  const int rem = (int)(i - b * S * S);
  const int qi = rem / S, ki = rem - qi * S;
  int qq = 0, qr = 0, kq = 0, kr = 0;
  if (qi >= kNumTok) {
    qq = (int)load_index(coords, cdtype, (b * npad + qi - kNumTok) * 2);
    qr = (int)load_index(coords, cdtype, (b * npad + qi - kNumTok) * 2 + 1);
  }
  int row;
  if (ki >= kNumTok) {
    kq = (int)load_index(coords, cdtype, (b * npad + ki - kNumTok) * 2);
    kr = (int)load_index(coords, cdtype, (b * npad + ki - kNumTok) * 2 + 1);
    if (load_mask(mask, mdtype, b * npad + ki - kNumTok) == 0.f) {
      out[i] = 237;
      return;
    }
  }
  row = pair_row(qi, ki, qq, qr, kq, kr, lut);
  out[i] = (uint8_t)row;
}

struct HeadsArgs {
  const __half* lnf16;    // (B*S, C): ln_final output (f16, the policy conv's input too), token + cell rows
  const float* rowmask;   // (B*S)
  int B, S, C;
  const float* vr_wT; const float* vr_b; const float* vh_wT; const float* vh_b;
  float* value_logits; float* value;
  const float* mr_wT; const float* mr_b; const float* mh_wT; const float* mh_b;
  float* ml_logits; float* ml;
  // serve reply (optional): legal-prefix softmax of each position's policy
  // logits written flat at prior_offs[b] (inference.py:998-1042)
  const float* policy;        // (B, npad) logits
  int npad;
  const int32_t* legal;       // (B) legal-prefix lengths
  const int64_t* prior_offs;  // (B) flat offsets
  float* priors;              // flat priors, or NULL (no reply)
  float* priors_logits;       // flat raw logits at the same offsets, or NULL
  // cell-mean chunk sums from pool_cells_kernel ([B][chunks][2][C] and
  // [B][chunks][2]), or NULL: the heads kernel pools the cells itself
  const float* pool;
  const float* pool_cnt;
};

// Masked cell mean (model.py:931-935) in a fixed order: a position's cell
// rows are cut into chunks of kPoolRows, each chunk into its even and odd
// rows; a (chunk, parity) unit adds its rows in row order, sixteen rows per
// batch of loads, and the unit sums of one parity are added in chunk order.
// The order depends only on the padded row count, so a position's mean is
// the same whether heads_kernel pools in place or adds the unit sums that
// pool_cells_kernel wrote, and whatever the rest of the batch is.
constexpr int kPoolRows = 128;  // a multiple of 32: no load batch crosses a chunk
constexpr int kPoolThreads = 128;
__host__ __device__ constexpr int pool_chunks(int npad) { return (npad + kPoolRows - 1) / kPoolRows; }

// Sum of rows n_begin, n_begin + 2, ... < n_end of one position (cell rows
// from `base`), channels 4 c4 .. 4 c4 + 3, and the sum of their mask values.
__device__ __forceinline__ float4 pool_unit(const __half* lnf16, const float* rowmask, long long base, int C, int c4,
                                            int n_begin, int n_end, float& cnt) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  cnt = 0.f;
  for (int n0 = n_begin; n0 < n_end; n0 += 32) {
    uint2 v[16];  // four f16 channels
    float mk[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int n = n0 + 2 * q;
      const bool in = n < n_end;
      mk[q] = in ? __ldg(rowmask + base + n) : 0.f;
      v[q] = in ? __ldg(reinterpret_cast<const uint2*>(lnf16 + (base + n) * C) + c4) : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v[q].x));
      const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v[q].y));
      s.x = fmaf(lo.x, mk[q], s.x);
      s.y = fmaf(lo.y, mk[q], s.y);
      s.z = fmaf(hi.x, mk[q], s.z);
      s.w = fmaf(hi.y, mk[q], s.w);
      cnt += mk[q];
    }
  }
  return s;
}

// The unit sums for batches whose heads_kernel CTAs would leave most SMs
// idle: one warp per (position, chunk, parity) unit, written to
// pool[unit][C] and pool_cnt[unit], unit = (b * chunks + chunk) * 2 + parity.
__global__ void __launch_bounds__(kPoolThreads) pool_cells_kernel(const __half* lnf16, const float* rowmask, int B,
                                                                  int S, int C, float* pool, float* pool_cnt) {
  pdl_launch_dependents();
  pdl_wait();  // ln_final and the row mask come from earlier kernels
  const int npad = S - kNumTok, nk = pool_chunks(npad);
  const long long unit = (long long)blockIdx.x * (kPoolThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (unit >= (long long)B * nk * 2) return;
  const int part = (int)(unit & 1);
  const long long bk = unit >> 1;
  const int b = (int)(bk / nk), k = (int)(bk - (long long)b * nk);
  const long long base = (long long)b * S + kNumTok;
  for (int c4 = lane; c4 < C / 4; c4 += 32) {
    float cnt;
    const float4 s = pool_unit(lnf16, rowmask, base, C, c4, k * kPoolRows + part, min(k * kPoolRows + kPoolRows, npad),
                               cnt);
    *reinterpret_cast<float4*>(pool + unit * C + 4 * c4) = s;
    if (c4 == lane && lane == 0) pool_cnt[unit] = cnt;
  }
}

constexpr int kHeadsThreads = 256;
constexpr int kHeadsKC = 32;  // layer-1 weight rows per shared-memory chunk

// softmax expectation over the 65 bins on linspace(-1, 1), clamped to [-1, 1]
// (losses.py:40-51).
__device__ __forceinline__ float decode_bins(const float* logits) {
  float mx = -INFINITY;
  for (int i = 0; i < kBins; ++i) mx = fmaxf(mx, logits[i]);
  float se = 0.f, sv = 0.f;
  for (int i = 0; i < kBins; ++i) {
    const float e = expf(logits[i] - mx);
    se += e;
    sv += e * (-1.f + 2.f * (float)i / (float)(kBins - 1));
  }
  return fminf(fmaxf(sv / se, -1.f), 1.f);
}

// Shared memory of heads_kernel<P> in floats, laid out as 16-byte aligned
// pieces: layer-1 weight ring [kHeadsRing][KC][C], inputs [3C][P], hidden
// [C][P], partial sums [max(2 P C, 3 * 65 * P, ns * C * P)], counts [2 P],
// logits [P][65].
constexpr int kHeadsRing = 4;  // weight chunks in flight per CTA
__host__ __device__ constexpr int heads_max(int x, int y) { return x > y ? x : y; }
__host__ __device__ constexpr int heads_red_floats(int C, int P) {
  return heads_max(heads_max(2 * P * C, 3 * kBins * P), heads_max(kHeadsThreads / C, 1) * C * P);
}
__host__ __device__ constexpr int heads_smem_floats(int C, int P) {
  return kHeadsRing * kHeadsKC * C + 3 * C * P + C * P + heads_red_floats(C, P) + 2 * P + P * kBins;
}

// Value (and moves-left) heads over cat(token a, token b, masked mean of the
// cells) of ln_final (model.py:931-1003): value_head(relu(value_reduction(.))),
// then the binned decode (losses.py:40-61). One CTA = P positions, 256
// threads; activations are kept position-minor in shared memory ([k][p]) so
// one 16-byte load gives four positions. The kernel runs once per forward, at
// MCTS batch sizes too, so it is built for latency: pooling gives each warp
// half of one position's rows and loads them in batches of 16 before adding
// them (or adds the unit sums of pool_cells_kernel, when a small batch of
// long positions ran it first); the layer-1 weights stream through a ring of cp.async chunks (three
// in flight while one is used); the dot products are split over K across
// thread groups and reduced in a fixed order.
template <int P>
__device__ void heads_pass(const HeadsArgs& a, int pass, float* sm, int b0, int npos) {
  const int C = a.C, S = a.S, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = 3 * C;
  float* wbuf = sm;                              // [ring][KC][C]
  float* vin = wbuf + kHeadsRing * kHeadsKC * C; // [3C][P]
  float* hidden = vin + 3 * C * P;               // [C][P]
  float* red = hidden + C * P;                   // partial sums
  float* redc = red + heads_red_floats(C, P);    // [2P] row counts of the pooling units
  float* logits = redc + 2 * P;                  // [P][65]
  const float* w1 = pass == 0 ? a.vr_wT : a.mr_wT;
  const float* b1 = pass == 0 ? a.vr_b : a.mr_b;
  const float* w2 = pass == 0 ? a.vh_wT : a.mh_wT;
  const float* b2 = pass == 0 ? a.vh_b : a.mh_b;
  const int nchunks = K / kHeadsKC;  // C is a multiple of 32, so K is a multiple of KC
  auto load_chunk = [&](int ch) {
    if (ch < nchunks) {
      const float* src = w1 + (long long)ch * kHeadsKC * C;
      float* dst = wbuf + (ch % kHeadsRing) * kHeadsKC * C;
      for (int i = tid * 4; i < kHeadsKC * C; i += kHeadsThreads * 4) cp_async16(smem_u32(dst + i), src + i, 16u);
    }
    cp_async_commit();  // one group per chunk (empty past the end) keeps the wait count uniform
  };
  for (int ch = 0; ch < kHeadsRing - 1; ++ch) load_chunk(ch);  // in flight during pooling
  pdl_wait();  // ln_final and the row mask come from earlier kernels (weights do not)

  // ---- inputs: summary tokens (model.py:1005-1009) and the masked mean of
  // the cells (model.py:931-935) ------------------------------------------
  const int ta = pass == 0 ? 0 : 4;
  for (int idx = tid; idx < P * 2 * C; idx += kHeadsThreads) {
    const int c = idx / P, p = idx - c * P;  // consecutive threads: consecutive positions of one channel
    float v = 0.f;
    if (p < npos) v = __half2float(a.lnf16[((long long)(b0 + p) * S + ta + (c >= C ? 1 : 0)) * C + (c % C)]);
    vin[idx] = v;
  }
  if (pass == 0) {  // the cell mean is shared by both heads (kept in vin[2C, 3C))
    // unit u = (position u / 2, rows of parity u % 2), summed over the
    // chunks in the order pool_unit documents
    const int npad = S - kNumTok, nk = pool_chunks(npad);
    for (int u = warp; u < 2 * P; u += kHeadsThreads / 32) {
      const int p = u >> 1, part = u & 1;
      const bool live = p < npos;
      const long long base = (long long)(b0 + (live ? p : 0)) * S + kNumTok;
      for (int c4 = lane; c4 < C / 4; c4 += 32) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        float cnt = 0.f;
        if (live && a.pool) {
          const long long u0 = (long long)(b0 + p) * nk * 2 + part;
#pragma unroll 4
          for (int k = 0; k < nk; ++k) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(a.pool + (u0 + 2 * k) * C) + c4);
            s.x += t.x;
            s.y += t.y;
            s.z += t.z;
            s.w += t.w;
            cnt += __ldg(a.pool_cnt + u0 + 2 * k);
          }
        } else if (live) {
          for (int k = 0; k < nk; ++k) {
            float ck;
            const float4 t = pool_unit(a.lnf16, a.rowmask, base, C, c4, k * kPoolRows + part,
                                       min(k * kPoolRows + kPoolRows, npad), ck);
            s.x += t.x;
            s.y += t.y;
            s.z += t.z;
            s.w += t.w;
            cnt += ck;
          }
        }
        *reinterpret_cast<float4*>(red + u * C + 4 * c4) = s;
        if (c4 == lane && lane == 0) redc[u] = cnt;
      }
    }
    __syncthreads();
    for (int idx = tid; idx < P * C; idx += kHeadsThreads) {
      const int c = idx / P, p = idx - c * P;
      const float v = red[(2 * p) * C + c] + red[(2 * p + 1) * C + c];
      const float n = redc[2 * p] + redc[2 * p + 1];
      vin[(2 * C + c) * P + p] = v / fmaxf(n, 1.f);
    }
  }

  // ---- layer 1: hidden = relu(vin . W1 + b1), K split over `ns` groups -----
  const int ns = C <= kHeadsThreads ? kHeadsThreads / C : 1;
  const int j = tid % C, g1 = tid / C;
  const bool act1 = g1 < ns;
  float acc[P];
#pragma unroll
  for (int p = 0; p < P; ++p) acc[p] = 0.f;
  for (int ch = 0; ch < nchunks; ++ch) {
    load_chunk(ch + kHeadsRing - 1);  // into the slot freed at the end of the previous step
    cp_async_wait<kHeadsRing - 1>();  // chunk ch landed (this thread's copies) ...
    __syncthreads();                  // ... and everyone's; the pooled inputs are visible
    if (act1) {
      const float* wb = wbuf + (ch % kHeadsRing) * kHeadsKC * C;
      const float* vk = vin + ch * kHeadsKC * P;
#pragma unroll 4
      for (int kk = g1; kk < kHeadsKC; kk += ns) {
        const float w = wb[kk * C + j];
#pragma unroll
        for (int p = 0; p < P; p += 4) {
          const float4 v = *reinterpret_cast<const float4*>(vk + kk * P + p);
          acc[p] = fmaf(w, v.x, acc[p]);
          acc[p + 1] = fmaf(w, v.y, acc[p + 1]);
          acc[p + 2] = fmaf(w, v.z, acc[p + 2]);
          acc[p + 3] = fmaf(w, v.w, acc[p + 3]);
        }
      }
    }
    __syncthreads();  // slot ch % ring may be refilled
  }
  if (act1)
#pragma unroll
    for (int p = 0; p < P; ++p) red[(g1 * C + j) * P + p] = acc[p];
  __syncthreads();
  for (int idx = tid; idx < C * P; idx += kHeadsThreads) {
    const int jj = idx / P, p = idx - jj * P;
    float v = __ldg(b1 + jj);
    for (int g = 0; g < ns; ++g) v += red[(g * C + jj) * P + p];
    hidden[jj * P + p] = fmaxf(v, 0.f);
  }
  __syncthreads();

  // ---- layer 2: logits = hidden . W2 + b2, C split over 3 groups ------------
  {
    const int o = tid % kBins, g2 = tid / kBins;  // 3 groups of 65 threads
    if (g2 < 3) {
      float acc2[P];
#pragma unroll
      for (int p = 0; p < P; ++p) acc2[p] = 0.f;
#pragma unroll 4
      for (int jj = g2; jj < C; jj += 3) {
        const float w = __ldg(w2 + (long long)jj * kBins + o);
#pragma unroll
        for (int p = 0; p < P; p += 4) {
          const float4 h = *reinterpret_cast<const float4*>(hidden + jj * P + p);
          acc2[p] = fmaf(w, h.x, acc2[p]);
          acc2[p + 1] = fmaf(w, h.y, acc2[p + 1]);
          acc2[p + 2] = fmaf(w, h.z, acc2[p + 2]);
          acc2[p + 3] = fmaf(w, h.w, acc2[p + 3]);
        }
      }
#pragma unroll
      for (int p = 0; p < P; ++p) red[(g2 * kBins + o) * P + p] = acc2[p];
    }
  }
  __syncthreads();
  float* lo = pass == 0 ? a.value_logits : a.ml_logits;
  for (int idx = tid; idx < P * kBins; idx += kHeadsThreads) {
    const int p = idx / kBins, o = idx - p * kBins;
    const float v = __ldg(b2 + o) + red[o * P + p] + red[(kBins + o) * P + p] + red[(2 * kBins + o) * P + p];
    logits[idx] = v;
    if (p < npos) lo[(long long)b0 * kBins + idx] = v;
  }
  __syncthreads();
  // ---- binned decode: one warp per position ---------------------------------
  float* dec = pass == 0 ? a.value : a.ml;
  if (dec) {
    for (int p = warp; p < npos; p += kHeadsThreads / 32) {
      const float* l = logits + p * kBins;
      float mx = -INFINITY;
      for (int i = lane; i < kBins; i += 32) mx = fmaxf(mx, l[i]);
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float se = 0.f, sv = 0.f;
      for (int i = lane; i < kBins; i += 32) {
        const float e = expf(l[i] - mx);
        se += e;
        sv += e * (-1.f + 2.f * (float)i / (float)(kBins - 1));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        se += __shfl_xor_sync(0xffffffffu, se, o);
        sv += __shfl_xor_sync(0xffffffffu, sv, o);
      }
      if (lane == 0) {
        const float e = fminf(fmaxf(sv / se, -1.f), 1.f);
        dec[b0 + p] = pass == 0 ? e : (e + 1.f) * 0.5f * 209.f;
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // shared buffers are reused by the next pass
}

// One warp per position: softmax over the first legal[b] policy logits,
// written flat (with the raw logits when asked) at prior_offs[b].
__device__ void heads_priors(const HeadsArgs& a, int b0, int npos) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int p = warp; p < npos; p += kHeadsThreads / 32) {
    const int b = b0 + p;
    const int L = min(__ldg(a.legal + b), a.npad);
    const float* row = a.policy + (long long)b * a.npad;
    float mx = -INFINITY;
    for (int i = lane; i < L; i += 32) mx = fmaxf(mx, row[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.f;
    for (int i = lane; i < L; i += 32) se += expf(row[i] - mx);
#pragma unroll
    for (int o = 16; o; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    const long long off = __ldg(a.prior_offs + b);
    for (int i = lane; i < L; i += 32) {
      const float x = row[i];
      a.priors[off + i] = expf(x - mx) / se;
      if (a.priors_logits) a.priors_logits[off + i] = x;
    }
  }
}

template <int P>
__global__ void __launch_bounds__(kHeadsThreads) heads_kernel(const HeadsArgs a) {
  extern __shared__ __align__(16) float hsm[];
  pdl_launch_dependents();
  const int b0 = blockIdx.x * P;
  const int npos = min(P, a.B - b0);
  heads_pass<P>(a, 0, hsm, b0, npos);
  if (a.ml_logits) heads_pass<P>(a, 1, hsm, b0, npos);
  if (a.priors) heads_priors(a, b0, npos);  // policy logits come from an earlier kernel (after pdl_wait)
}

__global__ void decode_binned_kernel(const float* logits, int B, float scale, float offset, float* out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const float e = decode_bins(logits + (long long)b * kBins);
  out[b] = (e + offset) * scale;
}

// One warp per row: softmax over the first legal_counts[b] logits
// (inference.py:998-1042), written at row_offsets[b].
__global__ void legal_softmax_kernel(const float* policy, int B, int npad, const int32_t* legal,
                                     const int64_t* offs, float* out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= B) return;
  const int L = min(legal[warp], npad);
  const float* row = policy + (long long)warp * npad;
  float mx = -INFINITY;
  for (int i = lane; i < L; i += 32) mx = fmaxf(mx, row[i]);
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f;
  for (int i = lane; i < L; i += 32) s += expf(row[i] - mx);
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  float* dst = out + offs[warp];
  for (int i = lane; i < L; i += 32) dst[i] = expf(row[i] - mx) / s;
}

// (taps, Cin, Cout) fp32 -> f16 [Cout][Kpad] with per-tap channel padding.
__global__ void pack_conv_kernel(const float* w, int taps, int cin, int cin_pad, int cout, int kpad, __half* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)cout * kpad) return;
  const int n = (int)(i / kpad), k = (int)(i % kpad);
  const int t = k / cin_pad, c = k % cin_pad;
  float v = 0.f;
  if (t < taps && c < cin) v = w[((long long)t * cin + c) * cout + n];
  out[i] = __float2half_rn(v);
}

__global__ void pack_linear_kernel(const float* w, int n, int k, int kpad, __half* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n * kpad) return;
  const int r = (int)(i / kpad), c = (int)(i % kpad);
  out[i] = __float2half_rn(c < k ? w[(long long)r * k + c] : 0.f);
}

}  // namespace sb
