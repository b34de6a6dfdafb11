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
  int* err;
};

// One thread per cell: stage features (f16, padded to 16 channels), the
// absolute-row gather table (tap 0 = self, taps 1..6 = DIRECTIONS neighbours;
// reference trunk gather_idx, model.py:860-863), the row mask and int32 coords.
__global__ void prep_cells_kernel(const PrepArgs a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
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

// Token rows of the residual stream (learned tokens) and of the first
// attention block's LN1 input (precomputed per weights).
__global__ void init_tokens_kernel(const float* tokens, const __half* tokens_ln16, int B, int S, int C,
                                   float* seq32, __half* xa16) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)B * kNumTok * C;
  if (i >= total) return;
  const long long b = i / ((long long)kNumTok * C);
  const long long r = i - b * kNumTok * C;
  const long long row = b * S + r / C;
  const int c = (int)(r % C);
  seq32[row * C + c] = tokens[r];
  xa16[row * C + c] = tokens_ln16[r];
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
  const float* lnf32;     // (B*S, C): ln_final output, token + cell rows
  const float* rowmask;   // (B*S)
  int B, S, C;
  const float* vr_wT; const float* vr_b; const float* vh_wT; const float* vh_b;
  float* value_logits; float* value;
  const float* mr_wT; const float* mr_b; const float* mh_wT; const float* mh_b;
  float* ml_logits; float* ml;
};

constexpr int kHeadsPos = 16;     // positions per CTA
constexpr int kHeadsThreads = 256;

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

// Value (and moves-left) heads over cat(token a, token b, masked mean of the
// cells) of ln_final (model.py:931-1003): value_head(relu(value_reduction(.))),
// then the binned decode (losses.py:40-61). One CTA = kHeadsPos positions,
// 256 threads; activations are kept position-minor in shared memory
// ([k][position]) so one 16-byte load gives four positions.
// layer 1: thread t owns output channel t % C for 8 positions (t / C picks
// which 8); layer 2: (bin, 4 positions) per thread.
__device__ void heads_mlp(const float* vin, int C, const float* wT, const float* bias, const float* hwT,
                          const float* hbias, float* hidden, float* logits_s) {
  const int tid = threadIdx.x;
  const int K = 3 * C;
  const int groups = kHeadsPos / 8;  // 2 groups of 8 positions
  for (int w0 = tid; w0 < C * groups; w0 += kHeadsThreads) {
    const int j = w0 % C, g = w0 / C;
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
#pragma unroll 4
    for (int k = 0; k < K; ++k) {
      const float w = __ldg(wT + (long long)k * C + j);
      const float4 v0 = *reinterpret_cast<const float4*>(vin + k * kHeadsPos + g * 8);
      const float4 v1 = *reinterpret_cast<const float4*>(vin + k * kHeadsPos + g * 8 + 4);
      acc[0] = fmaf(w, v0.x, acc[0]);
      acc[1] = fmaf(w, v0.y, acc[1]);
      acc[2] = fmaf(w, v0.z, acc[2]);
      acc[3] = fmaf(w, v0.w, acc[3]);
      acc[4] = fmaf(w, v1.x, acc[4]);
      acc[5] = fmaf(w, v1.y, acc[5]);
      acc[6] = fmaf(w, v1.z, acc[6]);
      acc[7] = fmaf(w, v1.w, acc[7]);
    }
    const float bj = __ldg(bias + j);
#pragma unroll
    for (int q = 0; q < 8; ++q) hidden[j * kHeadsPos + g * 8 + q] = fmaxf(acc[q] + bj, 0.f);
  }
  __syncthreads();
  for (int w0 = tid; w0 < kBins * (kHeadsPos / 4); w0 += kHeadsThreads) {
    const int o = w0 % kBins, g = w0 / kBins;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int j = 0; j < C; ++j) {
      const float w = __ldg(hwT + (long long)j * kBins + o);
      const float4 h = *reinterpret_cast<const float4*>(hidden + j * kHeadsPos + g * 4);
      acc[0] = fmaf(w, h.x, acc[0]);
      acc[1] = fmaf(w, h.y, acc[1]);
      acc[2] = fmaf(w, h.z, acc[2]);
      acc[3] = fmaf(w, h.w, acc[3]);
    }
    const float bo = __ldg(hbias + o);
#pragma unroll
    for (int q = 0; q < 4; ++q) logits_s[(g * 4 + q) * kBins + o] = acc[q] + bo;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kHeadsThreads) heads_kernel(const HeadsArgs a) {
  extern __shared__ float hsm[];
  const int C = a.C;
  float* vin = hsm;                                   // [3C][P]  (k-major, position-minor)
  float* hidden = vin + 3 * C * kHeadsPos;            // [C][P]
  float* logits = hidden + C * kHeadsPos;             // [P][65]
  const int b0 = blockIdx.x * kHeadsPos;
  const int npos = min(kHeadsPos, a.B - b0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int npad = a.S - kNumTok;

  // pooled mean of ln_final cells (model.py:931-935): one warp per position,
  // four channels per lane per 16-byte load
  for (int p = warp; p < kHeadsPos; p += kHeadsThreads / 32) {
    const bool live = p < npos;
    const long long base = (long long)(b0 + (live ? p : 0)) * a.S + kNumTok;
    for (int c4 = lane * 4; c4 < C; c4 += 128) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      float cnt = 0.f;
      if (live) {
#pragma unroll 4
        for (int n = 0; n < npad; ++n) {
          const float mk = __ldg(a.rowmask + base + n);
          const float4 v = __ldg(reinterpret_cast<const float4*>(a.lnf32 + (base + n) * C + c4));
          s.x = fmaf(v.x, mk, s.x);
          s.y = fmaf(v.y, mk, s.y);
          s.z = fmaf(v.z, mk, s.z);
          s.w = fmaf(v.w, mk, s.w);
          cnt += mk;
        }
      }
      const float inv = 1.f / fmaxf(cnt, 1.f);
      vin[(2 * C + c4) * kHeadsPos + p] = s.x * inv;
      vin[(2 * C + c4 + 1) * kHeadsPos + p] = s.y * inv;
      vin[(2 * C + c4 + 2) * kHeadsPos + p] = s.z * inv;
      vin[(2 * C + c4 + 3) * kHeadsPos + p] = s.w * inv;
    }
  }
  const int passes = a.ml_logits ? 2 : 1;
  for (int pass = 0; pass < passes; ++pass) {
    const int ta = pass == 0 ? 0 : 4;  // summary-token rows of the head (model.py:1005-1009)
    for (int idx = tid; idx < kHeadsPos * 2 * C; idx += kHeadsThreads) {
      const int p = idx / (2 * C), c = idx - p * 2 * C;
      float v = 0.f;
      if (p < npos) {
        const long long row = (long long)(b0 + p) * a.S + ta + (c >= C ? 1 : 0);
        v = __ldg(a.lnf32 + row * C + (c % C));
      }
      vin[c * kHeadsPos + p] = v;
    }
    __syncthreads();
    if (pass == 0)
      heads_mlp(vin, C, a.vr_wT, a.vr_b, a.vh_wT, a.vh_b, hidden, logits);
    else
      heads_mlp(vin, C, a.mr_wT, a.mr_b, a.mh_wT, a.mh_b, hidden, logits);
    float* lo = pass == 0 ? a.value_logits : a.ml_logits;
    float* dec = pass == 0 ? a.value : a.ml;
    for (int idx = tid; idx < npos * kBins; idx += kHeadsThreads) lo[(long long)b0 * kBins + idx] = logits[idx];
    if (dec && tid < npos) {
      const float e = decode_bins(logits + tid * kBins);
      dec[b0 + tid] = pass == 0 ? e : (e + 1.f) * 0.5f * 209.f;
    }
    __syncthreads();
  }
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
