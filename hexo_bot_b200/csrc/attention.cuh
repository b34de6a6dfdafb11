// Relative-position-biased multi-head attention core:
//
//   O[b, q, h, :] = softmax_k( Q.K^T / sqrt(d) + bias(b, h, q, k) ) . V
//
// over the joint [tokens ; cells] sequence of one position, as computed by the
// reference's RelPosAttention (packages/shrimp/python/shrimp/model.py:448-492)
// with its per-pair bias row (model.py:677-760) or its fused Triton kernel
// (packages/shrimp/python/shrimp/_triton_attn.py:60-130).
//
// Bias sources:
//   BIAS_COORDS : row computed on the fly from the two cells' axial coords
//                 through the 35x35 clamped-offset LUT; token classes;
//                 dead (masked) cell keys are excluded exactly.
//   BIAS_PAIR   : row read from a precomputed (B, S, S) uint8 pair table
//                 (row 237 = the -3e4 pad row, as in _build_pair_u8).
//   BIAS_OFFSET : row read from one (S, S) int32 offset map shared by the
//                 batch (the standalone microbench).
//
// One CTA = (64-query block, head, position), four warps x 16 query rows.
// Keys/values stream through shared memory in 64-key blocks (cp.async double
// buffer); scores, the online softmax (fp32, exp2 domain) and P.V run on
// mma.sync m16n8k16 with fp32 accumulation.
#pragma once

#include "ptx.cuh"

namespace sb {

enum BiasMode : int { BIAS_COORDS = 0, BIAS_PAIR = 1, BIAS_OFFSET = 2 };

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  long long pos_stride;   // elements between positions (q, k, v)
  long long row_stride;   // elements between sequence rows (q, k, v)
  long long head_stride;  // elements between heads (q, k, v)
  void* out;
  long long out_pos_stride;
  long long out_row_stride;
  long long out_head_stride;
  int B, S, H, D, ntok;
  float scale_log2;       // log2(e) / sqrt(D)
  int mode;
  const float* table;     // [table_rows][H] additive bias values
  int table_rows;
  const int32_t* coords;  // BIAS_COORDS: [B][S - ntok][2]
  const float* keymask;   // BIAS_COORDS: [B][S] (1 = live key); nullptr = all live
  const uint8_t* lut;     // BIAS_COORDS: [35*35]
  const uint8_t* pair;    // BIAS_PAIR: [B][S][S]
  const int32_t* offset_map;  // BIAS_OFFSET: [S][S]
};

constexpr int kAttnThreads = 128;
constexpr int kAttnBlockQ = 64;
constexpr int kAttnBlockK = 64;
constexpr int kMaxTableRows = 1024;
constexpr int kLutW = 35;
constexpr int kLutM = 17;

template <int DP>
struct AttnSmem {
  static constexpr int kRowBytes = DP * 2 + 16;  // padded: conflict-free ldmatrix
  static constexpr int kTileBytes = kAttnBlockK * kRowBytes;
  // layout: K[2], V[2], key coords[2][64] int2, key live[2][64] float, table[kMaxTableRows], lut
  static constexpr int kOffK = 0;
  static constexpr int kOffV = 2 * kTileBytes;
  static constexpr int kOffCoord = 4 * kTileBytes;
  static constexpr int kOffLive = kOffCoord + 2 * kAttnBlockK * 8;
  static constexpr int kOffTable = kOffLive + 2 * kAttnBlockK * 4;
  static constexpr int kOffLut = kOffTable + kMaxTableRows * 4;
  static constexpr int kBytes = kOffLut + kLutW * kLutW + 15;
};

template <typename T, int DP>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
  using SM = AttnSmem<DP>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int qblk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S, D = a.D;
  const long long hoff = (long long)b * a.pos_stride + (long long)h * a.head_stride;
  const T* Q = reinterpret_cast<const T*>(a.q) + hoff;
  const T* Kg = reinterpret_cast<const T*>(a.k) + hoff;
  const T* Vg = reinterpret_cast<const T*>(a.v) + hoff;
  float* table_s = reinterpret_cast<float*>(smem + SM::kOffTable);
  uint8_t* lut_s = smem + SM::kOffLut;

  for (int i = tid; i < a.table_rows; i += kAttnThreads)
    table_s[i] = __ldg(a.table + (long long)i * a.H + h) * 1.4426950408889634f;  // log2 domain
  if (a.mode == BIAS_COORDS)
    for (int i = tid; i < kLutW * kLutW; i += kAttnThreads) lut_s[i] = __ldg(a.lut + i);

  // ---- query fragments (rows q0 + g, q0 + g + 8) ----
  const int q0 = qblk * kAttnBlockQ + warp * 16;
  const int qr[2] = {q0 + g, q0 + g + 8};
  constexpr int KS = DP / 16;
  uint32_t qa[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = qr[e & 1];
      const int col = ks * 16 + 2 * t4 + ((e >> 1) << 3);
      uint32_t val = 0;
      if (row < S && col < D) val = *reinterpret_cast<const uint32_t*>(Q + (long long)row * a.row_stride + col);
      qa[ks][e] = val;
    }
  }
  int qq[2] = {0, 0}, qrr[2] = {0, 0};
  bool qtok[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    qtok[i] = qr[i] < a.ntok;
    if (a.mode == BIAS_COORDS && !qtok[i] && qr[i] < S) {
      const int32_t* c = a.coords + ((long long)b * (S - a.ntok) + (qr[i] - a.ntok)) * 2;
      qq[i] = __ldg(c);
      qrr[i] = __ldg(c + 1);
    }
  }

  float o[DP / 8][4];
#pragma unroll
  for (int j = 0; j < DP / 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  const int nkb = (S + kAttnBlockK - 1) / kAttnBlockK;
  const int pieces = DP / 8;  // 16-byte pieces per row (padded)
  auto load_block = [&](int kb, int buf) {
    const uint32_t sK = smem_u32(smem + SM::kOffK + buf * SM::kTileBytes);
    const uint32_t sV = smem_u32(smem + SM::kOffV + buf * SM::kTileBytes);
    for (int i = tid; i < kAttnBlockK * pieces; i += kAttnThreads) {
      const int r = i / pieces, p = i - r * pieces;
      const int key = kb * kAttnBlockK + r;
      const bool in = key < S && p * 8 < D;
      const long long off = (long long)key * a.row_stride + p * 8;
      cp_async16(sK + r * SM::kRowBytes + p * 16, in ? (const void*)(Kg + off) : (const void*)Kg, in ? 16 : 0);
      cp_async16(sV + r * SM::kRowBytes + p * 16, in ? (const void*)(Vg + off) : (const void*)Vg, in ? 16 : 0);
    }
    int2* kc = reinterpret_cast<int2*>(smem + SM::kOffCoord) + buf * kAttnBlockK;
    float* kl = reinterpret_cast<float*>(smem + SM::kOffLive) + buf * kAttnBlockK;
    for (int r = tid; r < kAttnBlockK; r += kAttnThreads) {
      const int key = kb * kAttnBlockK + r;
      float live = key < S ? 1.f : 0.f;
      int2 c = make_int2(0, 0);
      if (key < S && key >= a.ntok) {
        if (a.keymask) live = __ldg(a.keymask + (long long)b * S + key);
        if (a.mode == BIAS_COORDS) {
          const int32_t* cp = a.coords + ((long long)b * (S - a.ntok) + (key - a.ntok)) * 2;
          c = make_int2(__ldg(cp), __ldg(cp + 1));
        }
      }
      kc[r] = c;
      kl[r] = live;
    }
  };

  load_block(0, 0);
  cp_async_commit();
  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) load_block(kb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const uint32_t sK = smem_u32(smem + SM::kOffK + buf * SM::kTileBytes);
    const uint32_t sV = smem_u32(smem + SM::kOffV + buf * SM::kTileBytes);
    const int2* kc = reinterpret_cast<const int2*>(smem + SM::kOffCoord) + buf * kAttnBlockK;
    const float* kl = reinterpret_cast<const float*>(smem + SM::kOffLive) + buf * kAttnBlockK;

    // S = Q K^T for 8 key tiles of 8
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t kbf[2];
        const int l = lane & 15;
        const uint32_t addr = sK + (j * 8 + (l & 7)) * SM::kRowBytes + (ks * 16 + ((l >> 3) << 3)) * 2;
        ldmatrix_x2(kbf, addr);
        MmaTraits<T>::mma(s[j], qa[ks], kbf);
      }
    }
    // scale + bias + masks, row maxima
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = e >> 1;
        const int kloc = j * 8 + 2 * t4 + (e & 1);
        const int key = kb * kAttnBlockK + kloc;
        float val = -INFINITY;
        if (kl[kloc] != 0.f) {
          int row;
          if (a.mode == BIAS_COORDS) {
            const bool ktok = key < a.ntok;
            if (qtok[ri]) {
              row = ktok ? 236 : 235;
            } else if (ktok) {
              row = 234;
            } else {
              const int2 c = kc[kloc];
              const int dq = min(max(c.x - qq[ri], -kLutM), kLutM);
              const int dr = min(max(c.y - qrr[ri], -kLutM), kLutM);
              row = lut_s[(dq + kLutM) * kLutW + dr + kLutM];
            }
          } else if (a.mode == BIAS_PAIR) {
            row = qr[ri] < S ? __ldg(a.pair + ((long long)b * S + qr[ri]) * S + key) : 0;
            row = min(row, a.table_rows - 1);
          } else {
            row = qr[ri] < S ? __ldg(a.offset_map + (long long)qr[ri] * S + key) : 0;
            row = min(max(row, 0), a.table_rows - 1);
          }
          val = fmaf(s[j][e], a.scale_log2, table_s[row]);
        }
        s[j][e] = val;
        mx[ri] = fmaxf(mx[ri], val);
      }
    }
    float alpha[2];
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
      const float mnew = fmaxf(mrow[ri], mx[ri]);
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      alpha[ri] = exp2f(mrow[ri] - mref);
      mrow[ri] = mnew;
      mx[ri] = mref;
      lrow[ri] *= alpha[ri];
    }
#pragma unroll
    for (int jd = 0; jd < DP / 8; ++jd) {
      o[jd][0] *= alpha[0];
      o[jd][1] *= alpha[0];
      o[jd][2] *= alpha[1];
      o[jd][3] *= alpha[1];
    }
    // P = exp2(s - m), accumulate l, and P.V
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[e] = exp2f(s[j][e] - mx[e >> 1]);
        lrow[e >> 1] += p[e];
      }
      const int i = j >> 1, hi = j & 1;
      pa[i][hi ? 2 : 0] = MmaTraits<T>::pack(p[0], p[1]);
      pa[i][hi ? 3 : 1] = MmaTraits<T>::pack(p[2], p[3]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int jd = 0; jd < DP / 8; ++jd) {
        if (jd * 8 >= D) break;
        uint32_t vb[2];
        const int l = lane & 15;
        const uint32_t addr = sV + (i * 16 + (l & 7) + ((l >> 3) << 3)) * SM::kRowBytes + jd * 16;
        ldmatrix_x2_trans(vb, addr);
        MmaTraits<T>::mma(o[jd], pa[i], vb);
      }
    }
    __syncthreads();
  }
  cp_async_wait_all();

  // normalise and store
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    float l = lrow[ri];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    lrow[ri] = l > 0.f ? 1.f / l : 0.f;
  }
  T* O = reinterpret_cast<T*>(a.out) + (long long)b * a.out_pos_stride + (long long)h * a.out_head_stride;
#pragma unroll
  for (int jd = 0; jd < DP / 8; ++jd) {
    const int col = jd * 8 + 2 * t4;
    if (col >= D) break;
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      const int row = qr[ri];
      if (row >= S) continue;
      const uint32_t packed = MmaTraits<T>::pack(o[jd][2 * ri] * lrow[ri], o[jd][2 * ri + 1] * lrow[ri]);
      *reinterpret_cast<uint32_t*>(O + (long long)row * a.out_row_stride + col) = packed;
    }
  }
}

}  // namespace sb
