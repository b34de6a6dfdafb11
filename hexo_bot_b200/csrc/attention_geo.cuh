// Biased multi-head attention core for positions that share their geometry.
//
//   O[b, q, h, :] = softmax_k( Q.K^T / sqrt(d) + bias(b, h, q, k) ) . V
//
// Same operator as attn_kernel in BIAS_COORDS mode (RelPosAttention,
// packages/shrimp/python/shrimp/model.py:448-492, with the per-pair bias row
// of model.py:677-760), specialised for head_dim 16 and sequences of at most
// 80 tokens (the 61-cell disk of the serve configuration: 8 tokens + 61 cells).
//
// The bias of a pair depends only on the position's geometry: the hex
// coordinates of its cells and which keys are live. In the fixed-support
// regime every position of a batch covers the same set of cells, only in a
// different row order (the support lists legal cells first, then stones, then
// the rest). Attention is equivariant under a permutation of the rows, so each
// CTA keeps the bias tensor of its heads for the last cell set it saw in shared memory
// ([head][query][key] in f16, pre-divided by the softmax scale, in that set's
// canonical row order: the cells sorted by coordinates) and, per position,
// only maps its rows onto the canonical order: a 35x35 coordinate window
// gives each cell its canonical index, and the MMA operands are then gathered in canonical order for free,
// because ldmatrix takes one row address per lane. The cache is rebuilt only
// when a position's cell set or key liveness differs (every position of a
// real-support batch: still correct, just slower). The bias enters the score
// MMA as its C operand, which removes the per-score row-table and bias-table
// lookups of the general kernel.
//
// Per CTA (two per SM, each owning one group of four heads, persistent over
// the positions: b = blockIdx.x / G, + gridDim.x / G, ... for G head groups):
//   * q, k and v of a position arrive by TMA as 64-column boxes of S rows
//     (128-byte swizzle), double buffered, so the next position streams in
//     while this one is computed;
//   * warps take (head, 16-query tile) tasks: scores by mma.sync m16n8k16
//     with the cached bias as accumulator input, one-pass softmax in the exp2
//     domain (all <= 80 keys live in registers), P.V plus a ones column (the
//     row sums come out of the same MMA), fp32 throughout;
//   * the cell coordinates and key liveness of the next position are loaded
//     during the current one (one cell per thread).
#pragma once

#include "attention.cuh"

namespace sb {

constexpr int kGeoD = 16;          // head_dim of this kernel
constexpr int kGeoHeads = 4;       // heads per CTA: one 64-column box of q, k and v
constexpr int kGeoWarps = 10;      // two (head, query-tile) tasks per warp at S = 69
constexpr int kGeoThreads = kGeoWarps * 32;
constexpr int kGeoMaxS = 80;

// Shared-memory carve-up (bytes from a 1024-aligned base).
struct AttnGeoLayout {
  int sp;         // query rows padded to 16
  int nj;         // 8-key tiles covering S
  int nk;         // nj * 8: keys per cached bias row
  int box_bytes;  // one 64-column box of sp rows
  int nbox;       // boxes of one position (q, k and v of the CTA's head group)
  int buf_bytes;  // one position
  int cache_off;  // f16 bias [kGeoHeads][S][nk]
  int table_off;  // f32 bias table [256][kGeoHeads] (row 255 = excluded key)
  int lut_off;    // u8 35x35 clamped-offset LUT
  int geo_off;    // canonical cell coordinates [2][80] i32, key liveness [80] f32,
                  // coordinate window [35*35] u8, canonical index -> row [80] u8,
                  // scratch coordinates [2][80] i32
  int bar_off;    // two mbarriers
  int total;      // including the slack that aligns the dynamic base
};

__host__ __device__ inline AttnGeoLayout attn_geo_layout(int S) {
  AttnGeoLayout L{};
  L.sp = attn_pad16(S);
  L.nj = (S + 7) / 8;
  L.nk = L.nj * 8;
  L.box_bytes = L.sp * 128;
  L.nbox = 3;
  L.buf_bytes = L.nbox * L.box_bytes;
  L.cache_off = 2 * L.buf_bytes;
  L.table_off = L.cache_off + attn_round16(kGeoHeads * S * L.nk * 2);
  L.lut_off = L.table_off + 256 * kGeoHeads * 4;
  L.geo_off = L.lut_off + attn_round16(kLutW * kLutW);
  L.bar_off = L.geo_off + 2 * kGeoMaxS * 4 + kGeoMaxS * 4 + attn_round16(kLutW * kLutW) + kGeoMaxS +
              2 * kGeoMaxS * 4;
  L.total = L.bar_off + 16 + 1024;
  return L;
}

// mma.sync m16n8k16 with fp32 accumulation, as a pure register operation (no
// volatile: the compiler may interleave it with the softmax arithmetic).
template <typename T>
__device__ __forceinline__ void geo_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void geo_mma<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void geo_mma<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                       uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ uint32_t geo_one2();
template <>
__device__ __forceinline__ uint32_t geo_one2<__half>() { return 0x3C003C00u; }  // (1.0, 1.0) in f16
template <>
__device__ __forceinline__ uint32_t geo_one2<__nv_bfloat16>() { return 0x3F803F80u; }  // (1.0, 1.0) in bf16

// Byte address of (row r, 16-byte chunk c) in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t geo_swz(uint32_t box, int r, int c) {
  return box + r * 128 + ((c ^ (r & 7)) << 4);
}

// Requirements (checked by the host): mode BIAS_COORDS, D == 16, H a multiple
// of 4 (whole 64-column boxes), S <= 80, table_rows <= 255, q/k/v the three
// column blocks of one (B*S, 3*H*16) row-major buffer (tmap covers it with a
// {64, S} box), err may be null.
// NJ = ceil(S / 8) is a template parameter so the score, softmax and P.V
// loops unroll completely without tail branches.
template <typename T, int NJ>
__global__ void __launch_bounds__(kGeoThreads, 2)
    attn_geo_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int S = a.S, H = a.H, ntok = a.ntok, ncell = S - ntok;
  const AttnGeoLayout L = attn_geo_layout(S);
  const int QT = L.sp / 16, NK = L.nk;  // NK == 8 * NJ
  // head group of this CTA (four heads = one 64-column box of each of q, k, v);
  // the CTAs of a group stride over the positions
  const int G = H / kGeoHeads;
  const int gi = blockIdx.x % G;
  const int b0 = blockIdx.x / G, pstride = gridDim.x / G;
  __half* cache = reinterpret_cast<__half*>(gb + L.cache_off);
  float* table_s = reinterpret_cast<float*>(gb + L.table_off);
  uint8_t* lut_s = gb + L.lut_off;
  int32_t* ccache = reinterpret_cast<int32_t*>(gb + L.geo_off);        // canonical cell coordinates
  float* lcache = reinterpret_cast<float*>(ccache + 2 * kGeoMaxS);      // canonical key liveness
  uint8_t* slot = reinterpret_cast<uint8_t*>(lcache + kGeoMaxS);        // window -> canonical cell (255: none)
  uint8_t* rowof = slot + attn_round16(kLutW * kLutW);                  // canonical index -> row
  int32_t* tmpc = reinterpret_cast<int32_t*>(rowof + kGeoMaxS);         // this position's coordinates
  const uint32_t full0 = base + L.bar_off;

  // ---- once per CTA: bias table (pre-divided by the softmax scale; rows past
  // the table, including the excluded-key row 255, are -inf), LUT, zero pad
  // rows of every box, barriers --------------------------------------------
  pdl_launch_dependents();
  const float inv_scale = sqrtf((float)a.D);
  for (int i = tid; i < 256 * kGeoHeads; i += kGeoThreads) {
    const int r = i / kGeoHeads, hl = i - r * kGeoHeads;
    table_s[i] =
        r < a.table_rows ? __ldg(a.table + (long long)r * H + gi * kGeoHeads + hl) * inv_scale : -INFINITY;
  }
  for (int i = tid; i < kLutW * kLutW; i += kGeoThreads) lut_s[i] = __ldg(a.lut + i);
  {
    const int pad16 = (L.sp - S) * 8;  // 16-byte pieces of the pad rows of one box
    for (int i = tid; i < 2 * L.nbox * pad16; i += kGeoThreads) {
      const int bx = i / pad16, p = i - bx * pad16;
      *reinterpret_cast<uint4*>(gb + bx * L.box_bytes + S * 128 + p * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  if (tid == 0) {
    mbar_init(full0, 1);
    mbar_init(full0 + 8, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    prefetch_tmap(&tmap);
  }
  __syncthreads();
  pdl_wait();  // q, k, v, coordinates and the key mask come from earlier kernels

  auto issue = [&](int b, int buf) {  // thread 0
    const uint32_t bar = full0 + 8 * buf;
    mbar_arrive_expect_tx(bar, (uint32_t)(L.nbox * S * 128));
    const uint32_t dst = base + buf * L.buf_bytes;
    // q, k, v boxes of the group's heads: columns x * C + gi * 64
    for (int x = 0; x < L.nbox; ++x)
      tma_load_2d(dst + x * L.box_bytes, &tmap, x * H * kGeoD + gi * 64, b * S, bar);
  };
  // this thread's cell (row ntok + tid) of position b: coordinates, liveness
  struct GeoCell {
    int q, r;
    float live;
  };
  auto load_cell = [&](int b) {
    GeoCell c{0, 0, 1.f};
    if (tid < ncell) {
      c.q = __ldg(a.coords + ((long long)b * ncell + tid) * 2);
      c.r = __ldg(a.coords + ((long long)b * ncell + tid) * 2 + 1);
      if (a.keymask) c.live = __ldg(a.keymask + (long long)b * S + ntok + tid);
    }
    return c;
  };
  // Bias of every (head, query, key) for the cached geometry, in the row
  // classes of model.py:677-716: token->token 236, token->cell 235,
  // cell->token 234, cell->cell the clamped-offset LUT; keys that are dead or
  // past S are excluded (-inf).
  auto build_cache = [&]() {
    const int32_t* cc = ccache;
    for (int i = tid; i < S * NK; i += kGeoThreads) {
      const int q = i / NK, k = i - q * NK;
      int row = kRowExcluded;
      if (k < S && (k < ntok || lcache[k] != 0.f)) {
        if (q < ntok) {
          row = k < ntok ? 236 : 235;
        } else if (k < ntok) {
          row = 234;
        } else {
          const int dq = min(max(cc[2 * (k - ntok)] - cc[2 * (q - ntok)], -kLutM), kLutM);
          const int dr = min(max(cc[2 * (k - ntok) + 1] - cc[2 * (q - ntok) + 1], -kLutM), kLutM);
          row = lut_s[(dq + kLutM) * kLutW + dr + kLutM];
        }
      }
      const float* tr = table_s + row * kGeoHeads;
      __half* dst = cache + (long long)q * NK + k;
#pragma unroll
      for (int hl = 0; hl < kGeoHeads; ++hl) dst[(long long)hl * S * NK] = __float2half_rn(tr[hl]);
    }
  };

  if (tid == 0) {
    if (b0 < a.B) issue(b0, 0);
    if (b0 + pstride < a.B) issue(b0 + pstride, 1);
  }
  bool have = false;
  bool ok = true;
  int oq = 0, orr = 0;  // window origin: canonical cell 0
  GeoCell nxt = load_cell(b0 < a.B ? b0 : 0);
  const float c2 = a.scale_log2;  // scores here are Q.K + bias * sqrt(d); exp2 argument = (s - m) * c2
  const uint32_t one2 = geo_one2<T>();
  int j = 0;
  for (int b = b0; b < a.B; b += pstride, ++j) {
    const GeoCell cur = nxt;
    if (b + pstride < a.B) nxt = load_cell(b + pstride);  // in flight during this position
    // map this position's cells onto the cached canonical order
    bool miss = !have;
    int canon = -1;
    if (have && tid < ncell) {
      const int dq = cur.q - oq + kLutM, dr = cur.r - orr + kLutM;
      if (dq < 0 || dq >= kLutW || dr < 0 || dr >= kLutW) {
        miss = true;
      } else {
        const int c = slot[dq * kLutW + dr];
        if (c == 255 || lcache[ntok + c] != cur.live) {
          miss = true;
        } else {
          canon = c;
          rowof[ntok + c] = (uint8_t)(ntok + tid);
        }
      }
    }
    __syncthreads();
    // two rows with the same coordinates would leave a canonical index unmapped
    if (canon >= 0 && rowof[ntok + canon] != ntok + tid) miss = true;
    if (__syncthreads_or(miss)) {
      // rebuild. The canonical order of a cell set is its cells sorted by
      // (q, r) (row index as the tie-break), so a position's result does not
      // depend on which positions its CTA saw before.
      if (tid < ncell) {
        tmpc[2 * tid] = cur.q;
        tmpc[2 * tid + 1] = cur.r;
      }
      if (tid < ntok) lcache[tid] = 1.f;
      for (int i = tid; i < kLutW * kLutW; i += kGeoThreads) slot[i] = 255;
      for (int i = tid; i < L.sp; i += kGeoThreads) rowof[i] = (uint8_t)i;  // tokens and padding
      __syncthreads();
      int rank = 0;
      if (tid < ncell) {
        for (int jc = 0; jc < ncell; ++jc) {
          const int qj = tmpc[2 * jc], rj = tmpc[2 * jc + 1];
          rank += (qj < cur.q || (qj == cur.q && (rj < cur.r || (rj == cur.r && jc < tid)))) ? 1 : 0;
        }
        ccache[2 * rank] = cur.q;
        ccache[2 * rank + 1] = cur.r;
        lcache[ntok + rank] = cur.live;
        rowof[ntok + rank] = (uint8_t)(ntok + tid);
      }
      __syncthreads();
      oq = ccache[0];
      orr = ccache[1];
      if (tid < ncell) {
        const int dq = cur.q - oq + kLutM, dr = cur.r - orr + kLutM;
        if (dq >= 0 && dq < kLutW && dr >= 0 && dr < kLutW) slot[dq * kLutW + dr] = (uint8_t)rank;
      }
      build_cache();
      __syncthreads();
      have = true;
    }
    const int buf = j & 1;
    const bool got = mbar_wait(full0 + 8 * buf, (j >> 1) & 1);
    if (!__syncthreads_and(got)) {
      ok = false;
      break;
    }
    const uint32_t sbuf = base + buf * L.buf_bytes;
    T* Ob = reinterpret_cast<T*>(a.out) + (long long)b * a.out_pos_stride;
    // This lane's K and V row of every 16-key block (canonical order), as the
    // row's byte offset with its swizzle phase in bits 4-6: the ldmatrix address
    // of chunk c is then box + (ro ^ (c << 4)) (see geo_swz).
    uint32_t kro[(NJ + 1) / 2], vro[(NJ + 1) / 2];
#pragma unroll
    for (int j2 = 0; j2 < (NJ + 1) / 2; ++j2) {
      const int rk = rowof[j2 * 16 + (lane & 7) + ((lane >> 4) << 3)];
      const int rv = rowof[j2 * 16 + (lane & 7) + (((lane >> 3) & 1) << 3)];
      kro[j2] = rk * 128 + ((rk & 7) << 4);
      vro[j2] = rv * 128 + ((rv & 7) << 4);
    }

    for (int task = warp; task < kGeoHeads * QT; task += kGeoWarps) {
      const int hl = task / QT, qt = task - hl * QT;
      const int h = gi * kGeoHeads + hl;  // head index in the layer
      const int cq = hl * 2;              // first 16-byte chunk of the head inside its box
      const uint32_t sQ = sbuf;
      const uint32_t sK = sQ + L.box_bytes;
      const uint32_t sV = sK + L.box_bytes;
      uint32_t qa[4];
      ldmatrix_x4(qa, geo_swz(sQ, rowof[qt * 16 + (lane & 15)], cq + (lane >> 4)));
      // this thread's two query rows of the cached bias (padding queries read row S-1)
      const int q0 = min(qt * 16 + g, S - 1), q1 = min(qt * 16 + g + 8, S - 1);
      const __half2* bb0 = reinterpret_cast<const __half2*>(cache + ((long long)hl * S + q0) * NK + 2 * t4);
      const __half2* bb1 = reinterpret_cast<const __half2*>(cache + ((long long)hl * S + q1) * NK + 2 * t4);

      float s[NJ + 1][4];
#pragma unroll
      for (int jp = 0; jp < (NJ + 1) / 2; ++jp) {
        {
          uint32_t kb[4];
          ldmatrix_x4(kb, sK + (kro[jp] ^ ((uint32_t)(cq + ((lane >> 3) & 1)) << 4)));
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int jt = 2 * jp + u;
            if (jt < NJ) {
              const float2 f0 = __half22float2(bb0[jt * 4]);
              const float2 f1 = __half22float2(bb1[jt * 4]);
              s[jt][0] = f0.x;
              s[jt][1] = f0.y;
              s[jt][2] = f1.x;
              s[jt][3] = f1.y;
              geo_mma<T>(s[jt], qa, kb[2 * u], kb[2 * u + 1]);
            } else {
              s[jt][0] = s[jt][1] = s[jt][2] = s[jt][3] = -INFINITY;
            }
          }
        }
      }
      float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
      for (int jt = 0; jt < NJ; ++jt) {
        m0 = fmaxf(m0, fmaxf(s[jt][0], s[jt][1]));
        m1 = fmaxf(m1, fmaxf(s[jt][2], s[jt][3]));
      }
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
      const float n0 = m0 == -INFINITY ? 0.f : -m0 * c2;
      const float n1 = m1 == -INFINITY ? 0.f : -m1 * c2;

      float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f}, os[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < (NJ + 1) / 2; ++kk) {
        {
          uint32_t pa[4];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int jt = 2 * kk + u;
            if (jt < NJ) {
              const float p0 = ex2_approx(fmaf(s[jt][0], c2, n0));
              const float p1 = ex2_approx(fmaf(s[jt][1], c2, n0));
              const float p2 = ex2_approx(fmaf(s[jt][2], c2, n1));
              const float p3 = ex2_approx(fmaf(s[jt][3], c2, n1));
              pa[2 * u] = MmaTraits<T>::pack(p0, p1);
              pa[2 * u + 1] = MmaTraits<T>::pack(p2, p3);
            } else {
              pa[2 * u] = pa[2 * u + 1] = 0u;  // the key tile past S (odd NJ)
            }
          }
          uint32_t vb[4];
          ldmatrix_x4_trans(vb, sV + (vro[kk] ^ ((uint32_t)(cq + (lane >> 4)) << 4)));
          geo_mma<T>(o0, pa, vb[0], vb[1]);
          geo_mma<T>(o1, pa, vb[2], vb[3]);
          geo_mma<T>(os, pa, one2, one2);
        }
      }
      // normalise by the row sums and store (canonical rows >= S are padding)
      const float i0 = __fdividef(1.f, os[0]), i1 = __fdividef(1.f, os[2]);  // row sums are >= 1
      const int r0 = qt * 16 + g, r1 = r0 + 8;
      T* oh = Ob + (long long)h * a.out_head_stride + 2 * t4;
      if (r0 < S) {
        T* p = oh + (long long)rowof[r0] * a.out_row_stride;
        *reinterpret_cast<uint32_t*>(p) = MmaTraits<T>::pack(o0[0] * i0, o0[1] * i0);
        *reinterpret_cast<uint32_t*>(p + 8) = MmaTraits<T>::pack(o1[0] * i0, o1[1] * i0);
      }
      if (r1 < S) {
        T* p = oh + (long long)rowof[r1] * a.out_row_stride;
        *reinterpret_cast<uint32_t*>(p) = MmaTraits<T>::pack(o0[2] * i1, o0[3] * i1);
        *reinterpret_cast<uint32_t*>(p + 8) = MmaTraits<T>::pack(o1[2] * i1, o1[3] * i1);
      }
    }
    __syncthreads();  // every warp is done with buffer `buf`
    if (tid == 0 && b + 2 * pstride < a.B) issue(b + 2 * pstride, buf);
  }
  if (!ok) {
    // a TMA wait gave up: report it, then give the copies still in flight one
    // more bounded wait so none lands in shared memory after the CTA exits
    if (tid == 0) {
      if (a.err) atomicOr(a.err, SB_DEV_ERR_TIMEOUT);
      const int b_last = b0 + (j + 1) * pstride;
      mbar_wait(full0 + 8 * (j & 1), (j >> 1) & 1);
      if (b_last < a.B) mbar_wait(full0 + 8 * ((j + 1) & 1), ((j + 1) >> 1) & 1);
    }
    __syncthreads();
  }
}

}  // namespace sb
