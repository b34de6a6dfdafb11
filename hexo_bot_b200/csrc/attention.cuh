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
// One CTA per position (all heads): the position's bias-row table (query x
// key, one byte per pair) is built once in shared memory and shared by every
// head; K and V of a group of heads are staged once through cp.async (rows
// padded by 16 bytes for conflict-free ldmatrix). Eight warps then take
// (head, 16-query tile) tasks: Q fragments come straight from global memory,
// scores, the online softmax (fp32, exp2 domain, 32-key blocks) and P.V run
// on mma.sync m16n8k16 with fp32 accumulation, and each warp writes its
// output rows directly.
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
  const int32_t* seq_lens;  // [B] live sequence length, or nullptr = S: keys beyond it are
                            // skipped and query rows beyond it are written as zeros (PAIR:
                            // the reference op's seq_lens; COORDS: rows [live cells | pad])
  const int32_t* offset_map;  // BIAS_OFFSET: [S][S]
  int own_geometry;           // BIAS_COORDS: positions do not share one cell set (no geometry cache)
  int group;              // heads staged per pass (set by the host)
  int* err;               // device status word (SB_DEV_ERR_* bits), or nullptr
};

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnBlockK = 32;     // keys per online-softmax step
constexpr int kMaxTableRows = 1024;
constexpr int kLutW = 35;
constexpr int kLutM = 17;
constexpr uint8_t kRowExcluded = 255;  // row-table sentinel: key excluded (-inf)

__host__ __device__ constexpr int attn_pad16(int s) { return (s + 15) / 16 * 16; }
__host__ __device__ constexpr int attn_row_bytes(int dp) { return dp * 2 + 16; }
__host__ __device__ constexpr int attn_round16(int x) { return (x + 15) / 16 * 16; }
// Bias-table columns kept per head: with a row table, 256 entries (entry 255
// = -inf, the excluded-key sentinel); otherwise the table's own row count.
__host__ __device__ constexpr int attn_table_cols(int table_rows) {
  return table_rows <= 255 ? 256 : (table_rows + 3) / 4 * 4;
}
// Dynamic shared memory of one CTA: Q, K and V of `group` heads (rows padded
// by 16 bytes), the u8 row table (tables of <= 255 rows), the key coordinates
// and liveness, the bias-table columns of the group, the LUT.
__host__ __device__ constexpr int attn_smem_bytes(int S, int dp, int group, int table_rows) {
  return 3 * group * attn_pad16(S) * attn_row_bytes(dp) +
         (table_rows <= 255 ? attn_round16(attn_pad16(S) * attn_pad16(S)) : 0) + attn_pad16(S) * 12 +
         group * attn_table_cols(table_rows) * 4 + attn_round16(kLutW * kLutW);
}

// 2^x on the special-function unit (ex2.approx: max relative error ~2^-22;
// 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Scores of one 16-query x 8-key tile plus bias, in the log2 domain.
// Row-table path: rt0 / rt1 point at the row-table rows of the thread's two
// queries; two consecutive keys share one 16-bit load.
template <typename T, int KS>
__device__ __forceinline__ void attn_score_tile(float (&out)[4], const uint32_t (&qa)[KS][4], uint32_t sK, int RB,
                                                int key0, int lane, float scale, const float* tab,
                                                const uint8_t* rt0, const uint8_t* rt1) {
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    uint32_t kbf[2];
    const int l = lane & 15;
    ldmatrix_x2(kbf, sK + (key0 + (l & 7)) * RB + (ks * 16 + ((l >> 3) << 3)) * 2);
    MmaTraits<T>::mma(acc, qa[ks], kbf);
  }
  const int kc = key0 + 2 * (lane & 3);
  const uint32_t r0 = *reinterpret_cast<const uint16_t*>(rt0 + kc);
  const uint32_t r1 = *reinterpret_cast<const uint16_t*>(rt1 + kc);
  out[0] = fmaf(acc[0], scale, tab[r0 & 255u]);
  out[1] = fmaf(acc[1], scale, tab[r0 >> 8]);
  out[2] = fmaf(acc[2], scale, tab[r1 & 255u]);
  out[3] = fmaf(acc[3], scale, tab[r1 >> 8]);
}

// Persistent: CTA c handles positions c, c + grid, ... The LUT (and the bias
// table when all heads fit in one group) are loaded once per CTA. NT = key
// tiles of 8 per softmax step: 10 (one pass, sequences <= 80) or 4 (online
// softmax over 32-key blocks).
template <typename T, int DP, int NT>
__global__ void __launch_bounds__(kAttnThreads, 2) attn_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int S = a.S, D = a.D, G = a.group;
  const int SP = attn_pad16(S);
  constexpr int RB = attn_row_bytes(DP);
  constexpr int KB = NT * 8;
  const bool use_rowtab = a.table_rows <= 255;
  const int tcols = attn_table_cols(a.table_rows);
  const int tile_bytes = G * SP * RB;  // one of Q / K / V

  uint8_t* qkv_s = smem;                                             // Q [G][SP][RB], K, V
  uint8_t* rowtab = smem + 3 * tile_bytes;                           // [SP][SP]
  int2* kcoord = reinterpret_cast<int2*>(rowtab + (use_rowtab ? attn_round16(SP * SP) : 0));  // [SP]
  float* klive = reinterpret_cast<float*>(kcoord + SP);              // [SP]
  float* table_s = klive + SP;                                       // [G][tcols]
  uint8_t* lut_s = reinterpret_cast<uint8_t*>(table_s + G * tcols);

  if (a.mode == BIAS_COORDS)
    for (int i = tid; i < kLutW * kLutW; i += kAttnThreads) lut_s[i] = __ldg(a.lut + i);
  auto load_table = [&](int h0, int gh) {
    for (int i = tid; i < gh * tcols; i += kAttnThreads) {
      const int hl = i / tcols, r = i - hl * tcols;
      float v = -INFINITY;  // entries past the table: the excluded sentinel
      if (r < a.table_rows) v = __ldg(a.table + (long long)r * a.H + h0 + hl) * 1.4426950408889634f;
      table_s[i] = v;
    }
  };
  const bool one_group = G >= a.H;
  if (one_group) load_table(0, a.H);

  constexpr int PPR = DP / 8;  // 16-byte pieces per (row, head)
  constexpr int KS = DP / 16;
  const int QT = SP / 16;

  for (int b = blockIdx.x; b < a.B; b += gridDim.x) {
    const T* Qb = reinterpret_cast<const T*>(a.q) + (long long)b * a.pos_stride;
    const T* Kb = reinterpret_cast<const T*>(a.k) + (long long)b * a.pos_stride;
    const T* Vb = reinterpret_cast<const T*>(a.v) + (long long)b * a.pos_stride;
    T* Ob = reinterpret_cast<T*>(a.out) + (long long)b * a.out_pos_stride;
    int n_keys = S;
    if (a.seq_lens) n_keys = max(0, min(S, __ldg(a.seq_lens + b)));

    // stage Q, K, V of heads [h0, h0 + gh) (zero rows >= S, zero columns >= D)
    auto stage = [&](int h0, int gh) {
      const int total = SP * gh * PPR;
      for (int i = tid; i < total; i += kAttnThreads) {
        const int p = i % PPR, hl = (i / PPR) % gh, r = i / (PPR * gh);
        const bool in = r < S && p * 8 < D;
        const long long off = (long long)r * a.row_stride + (long long)(h0 + hl) * a.head_stride + p * 8;
        const uint32_t dq = smem_u32(qkv_s + (hl * SP + r) * RB + p * 16);
        cp_async16(dq, in ? (const void*)(Qb + off) : (const void*)Qb, in ? 16u : 0u);
        cp_async16(dq + tile_bytes, in ? (const void*)(Kb + off) : (const void*)Kb, in ? 16u : 0u);
        cp_async16(dq + 2 * tile_bytes, in ? (const void*)(Vb + off) : (const void*)Vb, in ? 16u : 0u);
      }
      cp_async_commit();
    };

    __syncthreads();  // the previous position's readers are done
    if (one_group) stage(0, a.H);  // in flight while the row table is built

    // ---- per-position bias-row table (shared by every head); keys that are
    // excluded or past the live length get the -inf sentinel ----------------
    if (use_rowtab) {
      if (a.mode == BIAS_COORDS) {
        const int32_t* cb = a.coords + (long long)b * (S - a.ntok) * 2;
        for (int k = tid; k < SP; k += kAttnThreads) {
          int2 c = make_int2(0, 0);
          float live = k < S ? 1.f : 0.f;
          if (k < S && k >= a.ntok) {
            c = make_int2(__ldg(cb + 2 * (k - a.ntok)), __ldg(cb + 2 * (k - a.ntok) + 1));
            if (a.keymask) live = __ldg(a.keymask + (long long)b * S + k);
          }
          kcoord[k] = c;
          klive[k] = live;
        }
        __syncthreads();
      }
      // rows across warps, keys across lanes (no division per entry): lane L
      // of warp w visits entries L, L + 32, ... of the rows w, w + 8, ...
      int qi = warp, ki = lane;
      while (ki >= SP) {
        ki -= SP;
        qi += kAttnWarps;
      }
      while (qi < SP) {
        const int i = qi * SP + ki;
        int row = kRowExcluded;
        if (ki < n_keys) {
          if (qi >= S) {
            row = 0;  // padding query rows: any finite row
          } else if (a.mode == BIAS_COORDS) {
            if (klive[ki] == 0.f) {
              row = kRowExcluded;
            } else if (qi < a.ntok) {
              row = ki < a.ntok ? 236 : 235;
            } else if (ki < a.ntok) {
              row = 234;
            } else {
              const int2 cq = kcoord[qi], ck = kcoord[ki];
              const int dq = min(max(ck.x - cq.x, -kLutM), kLutM);
              const int dr = min(max(ck.y - cq.y, -kLutM), kLutM);
              row = lut_s[(dq + kLutM) * kLutW + dr + kLutM];
            }
          } else if (a.mode == BIAS_PAIR) {
            row = min((int)__ldg(a.pair + ((long long)b * S + qi) * S + ki), a.table_rows - 1);
          } else {
            row = min(max(__ldg(a.offset_map + (long long)qi * S + ki), 0), a.table_rows - 1);
          }
        }
        rowtab[i] = (uint8_t)row;
        ki += 32;
        while (ki >= SP) {
          ki -= SP;
          qi += kAttnWarps;
        }
      }
    }

    for (int h0 = 0; h0 < a.H; h0 += G) {
      const int gh = min(G, a.H - h0);
      if (!one_group) {
        __syncthreads();  // previous group's readers are done
        stage(h0, gh);
        load_table(h0, gh);
      }
      cp_async_wait_all();
      __syncthreads();

      for (int task = warp; task < gh * QT; task += kAttnWarps) {
        const int hl = task / QT, qt = task - hl * QT;
        const int h = h0 + hl;
        const int qr[2] = {qt * 16 + g, qt * 16 + g + 8};
        const uint32_t sQ = smem_u32(qkv_s + hl * SP * RB);
        const uint32_t sK = sQ + tile_bytes;
        const uint32_t sV = sQ + 2 * tile_bytes;
        const float* tab = table_s + (one_group ? h : hl) * tcols;
        const uint8_t* rt0 = rowtab + qr[0] * SP;
        const uint8_t* rt1 = rowtab + qr[1] * SP;

        uint32_t qa[KS][4];
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          // x4: rows qt*16 + (lane & 15), 8-column half (lane >> 4)
          const uint32_t addr = sQ + (qt * 16 + (lane & 15)) * RB + (ks * 16 + ((lane >> 4) << 3)) * 2;
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                       : "=r"(qa[ks][0]), "=r"(qa[ks][1]), "=r"(qa[ks][2]), "=r"(qa[ks][3])
                       : "r"(addr));
        }

        float o[DP / 8][4];
#pragma unroll
        for (int j = 0; j < DP / 8; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
        float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

        // query tiles wholly past the live length do no work (written as zeros)
        const int key_end = qt * 16 < n_keys ? n_keys : 0;
        for (int k0 = 0; k0 < key_end; k0 += KB) {
          float s[NT][4];
          float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
          for (int j = 0; j < NT; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) s[j][e] = -INFINITY;
            if (k0 + j * 8 >= n_keys) continue;  // warp-uniform
            if (use_rowtab) {
              attn_score_tile<T, KS>(s[j], qa, sK, RB, k0 + j * 8, lane, a.scale_log2, tab, rt0, rt1);
            } else {
              float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int ks = 0; ks < KS; ++ks) {
                uint32_t kbf[2];
                const int l = lane & 15;
                ldmatrix_x2(kbf, sK + (k0 + j * 8 + (l & 7)) * RB + (ks * 16 + ((l >> 3) << 3)) * 2);
                MmaTraits<T>::mma(acc, qa[ks], kbf);
              }
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int qi = qr[e >> 1];
                const int ki = k0 + j * 8 + 2 * t4 + (e & 1);
                if (ki < n_keys) {
                  const int row =
                      qi < S ? min(max(__ldg(a.offset_map + (long long)qi * S + ki), 0), a.table_rows - 1) : 0;
                  s[j][e] = fmaf(acc[e], a.scale_log2, tab[row]);
                }
              }
            }
            mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
            mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
          }
#pragma unroll
          for (int ri = 0; ri < 2; ++ri) {
            mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
            mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
          }
          if (NT * 8 < 80 || k0 > 0) {  // online rescale (not needed for the single pass)
#pragma unroll
            for (int ri = 0; ri < 2; ++ri) {
              const float mnew = fmaxf(mrow[ri], mx[ri]);
              const float mref = mnew == -INFINITY ? 0.f : mnew;
              const float alpha = ex2_approx(mrow[ri] - mref);
              mrow[ri] = mnew;
              mx[ri] = mref;
              lrow[ri] *= alpha;
#pragma unroll
              for (int jd = 0; jd < DP / 8; ++jd) {
                o[jd][2 * ri] *= alpha;
                o[jd][2 * ri + 1] *= alpha;
              }
            }
          } else {
#pragma unroll
            for (int ri = 0; ri < 2; ++ri) {
              mrow[ri] = mx[ri];
              mx[ri] = mx[ri] == -INFINITY ? 0.f : mx[ri];
            }
          }
          uint32_t pa[(NT + 1) / 2][4];
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              p[e] = ex2_approx(s[j][e] - mx[e >> 1]);
              lrow[e >> 1] += p[e];
            }
            const int i = j >> 1, hi = j & 1;
            pa[i][hi ? 2 : 0] = MmaTraits<T>::pack(p[0], p[1]);
            pa[i][hi ? 3 : 1] = MmaTraits<T>::pack(p[2], p[3]);
          }
          if (NT & 1) {
            pa[NT / 2][2] = 0u;
            pa[NT / 2][3] = 0u;
          }
#pragma unroll
          for (int i = 0; i < (NT + 1) / 2; ++i) {
            if (k0 + i * 16 >= n_keys) break;  // warp-uniform; V rows beyond are never read
#pragma unroll
            for (int jd = 0; jd < DP / 8; ++jd) {
              if (jd * 8 >= D) break;
              uint32_t vb[2];
              const int l = lane & 15;
              ldmatrix_x2_trans(vb, sV + (k0 + i * 16 + (l & 7) + ((l >> 3) << 3)) * RB + jd * 16);
              MmaTraits<T>::mma(o[jd], pa[i], vb);
            }
          }
        }

        // normalise and store (rows >= the live length are written as zeros)
#pragma unroll
        for (int ri = 0; ri < 2; ++ri) {
          float l = lrow[ri];
          l += __shfl_xor_sync(0xffffffffu, l, 1);
          l += __shfl_xor_sync(0xffffffffu, l, 2);
          lrow[ri] = (l > 0.f && qr[ri] < n_keys) ? 1.f / l : 0.f;
        }
#pragma unroll
        for (int jd = 0; jd < DP / 8; ++jd) {
          const int col = jd * 8 + 2 * t4;
          if (col >= D) break;
#pragma unroll
          for (int ri = 0; ri < 2; ++ri) {
            const int row = qr[ri];
            if (row >= S) continue;
            const uint32_t packed = MmaTraits<T>::pack(o[jd][2 * ri] * lrow[ri], o[jd][2 * ri + 1] * lrow[ri]);
            *reinterpret_cast<uint32_t*>(Ob + (long long)row * a.out_row_stride + (long long)h * a.out_head_stride +
                                         col) = packed;
          }
        }
      }
    }
  }
}

// ---- long sequences ---------------------------------------------------------
// Sequences whose per-position row table or K/V do not fit in shared memory
// (real supports, hundreds to thousands of cells) use a streaming kernel: one
// CTA = (64-query block, head, position), four warps x 16 query rows, K/V in
// 64-key blocks through a cp.async double buffer, bias rows computed per pair
// on the fly (LUT in shared memory) or read from the pair / offset table.
constexpr int kStreamThreads = 128;
constexpr int kStreamBlockQ = 64;
constexpr int kStreamBlockK = 64;

// (1.0, 1.0) as a packed pair of T
template <typename T>
__device__ __forceinline__ uint32_t one_pair() {
  return std::is_same<T, __half>::value ? 0x3C003C00u : 0x3F803F80u;
}

template <int DP>
struct AttnStreamSmem {
  static constexpr int kRowBytes = DP * 2 + 16;  // padded: conflict-free ldmatrix
  static constexpr int kTileBytes = kStreamBlockK * kRowBytes;
  // layout: K[2], V[2], key coords[2][64] int2, key live[2][64] float, table[kMaxTableRows], lut
  static constexpr int kOffK = 0;
  static constexpr int kOffV = 2 * kTileBytes;
  static constexpr int kOffCoord = 4 * kTileBytes;
  static constexpr int kOffLive = kOffCoord + 2 * kStreamBlockK * 8;
  static constexpr int kOffTable = kOffLive + 2 * kStreamBlockK * 4;
  static constexpr int kOffLut = kOffTable + kMaxTableRows * 4;
  // BIAS_COORDS: the head's bias of every clamped offset, table[lut[dq][dr]] (log2 domain)
  static constexpr int kOffImg = (kOffLut + kLutW * kLutW + 15) / 16 * 16;
  static constexpr int kBytes = kOffImg + kLutW * kLutW * 4 + 15;
};

template <typename T, int DP>
__global__ void __launch_bounds__(kStreamThreads) attn_stream_kernel(const AttnArgs a) {
  using SM = AttnStreamSmem<DP>;
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int qblk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S, D = a.D;
  const long long hoff = (long long)b * a.pos_stride + (long long)h * a.head_stride;
  const T* Q = reinterpret_cast<const T*>(a.q) + hoff;
  const T* Kg = reinterpret_cast<const T*>(a.k) + hoff;
  const T* Vg = reinterpret_cast<const T*>(a.v) + hoff;
  const int n_live = a.seq_lens ? max(0, min(S, __ldg(a.seq_lens + b))) : S;
  // a query block wholly past the live length: zeros, no key pass
  if (qblk * kStreamBlockQ >= n_live) {
    T* Ob = reinterpret_cast<T*>(a.out) + (long long)b * a.out_pos_stride + (long long)h * a.out_head_stride;
    for (int i = tid; i < kStreamBlockQ * D; i += kStreamThreads) {
      const int row = qblk * kStreamBlockQ + i / D;
      if (row < S) reinterpret_cast<uint16_t*>(Ob)[(long long)row * a.out_row_stride + i % D] = 0;  // +0.0
    }
    return;
  }
  float* table_s = reinterpret_cast<float*>(smem + SM::kOffTable);
  uint8_t* lut_s = smem + SM::kOffLut;

  float* img_s = reinterpret_cast<float*>(smem + SM::kOffImg);
  for (int i = tid; i < a.table_rows; i += kStreamThreads)
    table_s[i] = __ldg(a.table + (long long)i * a.H + h) * 1.4426950408889634f;  // log2 domain
  if (a.mode == BIAS_COORDS)
    for (int i = tid; i < kLutW * kLutW; i += kStreamThreads) lut_s[i] = __ldg(a.lut + i);
  __syncthreads();
  // one lookup per cell pair: the head's bias of each clamped (dq, dr)
  if (a.mode == BIAS_COORDS)
    for (int i = tid; i < kLutW * kLutW; i += kStreamThreads) img_s[i] = table_s[min((int)lut_s[i], a.table_rows - 1)];
  // token rows of model.py:677-716: token->token 236, token->cell 235, cell->token 234
  const float b_tt = a.mode == BIAS_COORDS ? table_s[min(236, a.table_rows - 1)] : 0.f;
  const float b_tc = a.mode == BIAS_COORDS ? table_s[min(235, a.table_rows - 1)] : 0.f;
  const float b_ct = a.mode == BIAS_COORDS ? table_s[min(234, a.table_rows - 1)] : 0.f;

  // ---- query fragments (rows q0 + g, q0 + g + 8) ----
  const int q0 = qblk * kStreamBlockQ + warp * 16;
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
  // query coordinates shifted by the clamp radius: a key's image column is
  // clamp(kq - qq + M, 0, 2M), row clamp(kr - qr + M, 0, 2M)
  int qq[2] = {kLutM, kLutM}, qrr[2] = {kLutM, kLutM};
  bool qtok[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    qtok[i] = qr[i] < a.ntok;
    if (a.mode == BIAS_COORDS && !qtok[i] && qr[i] < S) {
      const int32_t* c = a.coords + ((long long)b * (S - a.ntok) + (qr[i] - a.ntok)) * 2;
      qq[i] = __ldg(c) - kLutM;
      qrr[i] = __ldg(c + 1) - kLutM;
    }
  }

  float o[DP / 8][4];
#pragma unroll
  for (int j = 0; j < DP / 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  // row sums of P come out of one more MMA per 16 keys, P times a ones tile
  // (rows g and g + 8 in elements 0 and 2), the same rounded P as the output
  float osum[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t ones2[2] = {one_pair<T>(), one_pair<T>()};

  const int nkb = (n_live + kStreamBlockK - 1) / kStreamBlockK;  // key blocks past the live length: skipped
  const int pieces = DP / 8;  // 16-byte pieces per row (padded)
  auto load_block = [&](int kb, int buf) {
    const uint32_t sK = smem_u32(smem + SM::kOffK + buf * SM::kTileBytes);
    const uint32_t sV = smem_u32(smem + SM::kOffV + buf * SM::kTileBytes);
    for (int i = tid; i < kStreamBlockK * pieces; i += kStreamThreads) {
      const int r = i / pieces, p = i - r * pieces;
      const int key = kb * kStreamBlockK + r;
      const bool in = key < S && p * 8 < D;
      const long long off = (long long)key * a.row_stride + p * 8;
      cp_async16(sK + r * SM::kRowBytes + p * 16, in ? (const void*)(Kg + off) : (const void*)Kg, in ? 16 : 0);
      cp_async16(sV + r * SM::kRowBytes + p * 16, in ? (const void*)(Vg + off) : (const void*)Vg, in ? 16 : 0);
    }
    int2* kc = reinterpret_cast<int2*>(smem + SM::kOffCoord) + buf * kStreamBlockK;
    float* kl = reinterpret_cast<float*>(smem + SM::kOffLive) + buf * kStreamBlockK;
    for (int r = tid; r < kStreamBlockK; r += kStreamThreads) {
      const int key = kb * kStreamBlockK + r;
      float live = key < n_live ? 1.f : 0.f;
      int2 c = make_int2(0, 0);
      if (key < S && key >= a.ntok) {
        if (a.keymask && key < n_live) live = __ldg(a.keymask + (long long)b * S + key);
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
    const int2* kc = reinterpret_cast<const int2*>(smem + SM::kOffCoord) + buf * kStreamBlockK;
    const float* kl = reinterpret_cast<const float*>(smem + SM::kOffLive) + buf * kStreamBlockK;

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
    // scale + bias + masks, row maxima. A block of live cell keys seen from
    // cell query rows (the bulk of a long sequence) takes a branch-free path.
    float mx[2] = {-INFINITY, -INFINITY};
    const bool cells_only = a.mode == BIAS_COORDS && kb * kStreamBlockK >= a.ntok &&
                            __syncthreads_and(tid >= kStreamBlockK || kl[tid] != 0.f) && q0 >= a.ntok;
    if (cells_only) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int ri = e >> 1;
          const int2 c = kc[j * 8 + 2 * t4 + (e & 1)];
          const int iq = min(max(c.x - qq[ri], 0), 2 * kLutM);
          const int ir = min(max(c.y - qrr[ri], 0), 2 * kLutM);
          const float val = fmaf(s[j][e], a.scale_log2, img_s[iq * kLutW + ir]);
          s[j][e] = val;
          mx[ri] = fmaxf(mx[ri], val);
        }
      }
    } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = e >> 1;
        const int kloc = j * 8 + 2 * t4 + (e & 1);
        const int key = kb * kStreamBlockK + kloc;
        float val = -INFINITY;
        if (kl[kloc] != 0.f) {
          float bias;
          if (a.mode == BIAS_COORDS) {
            const bool ktok = key < a.ntok;
            if (qtok[ri]) {
              bias = ktok ? b_tt : b_tc;
            } else if (ktok) {
              bias = b_ct;
            } else {
              const int2 c = kc[kloc];
              const int iq = min(max(c.x - qq[ri], 0), 2 * kLutM);
              const int ir = min(max(c.y - qrr[ri], 0), 2 * kLutM);
              bias = img_s[iq * kLutW + ir];
            }
          } else if (a.mode == BIAS_PAIR) {
            int row = qr[ri] < S ? __ldg(a.pair + ((long long)b * S + qr[ri]) * S + key) : 0;
            bias = table_s[min(row, a.table_rows - 1)];
          } else {
            int row = qr[ri] < S ? __ldg(a.offset_map + (long long)qr[ri] * S + key) : 0;
            bias = table_s[min(max(row, 0), a.table_rows - 1)];
          }
          val = fmaf(s[j][e], a.scale_log2, bias);
        }
        s[j][e] = val;
        mx[ri] = fmaxf(mx[ri], val);
      }
    }
    }
    float alpha[2];
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
      const float mnew = fmaxf(mrow[ri], mx[ri]);
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      alpha[ri] = ex2_approx(mrow[ri] - mref);
      mrow[ri] = mnew;
      mx[ri] = mref;
    }
    osum[0] *= alpha[0];
    osum[1] *= alpha[0];
    osum[2] *= alpha[1];
    osum[3] *= alpha[1];
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
      for (int e = 0; e < 4; ++e) p[e] = ex2_approx(s[j][e] - mx[e >> 1]);
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
      MmaTraits<T>::mma(osum, pa[i], ones2);
    }
    __syncthreads();
  }
  cp_async_wait_all();

  // normalise and store
  float lrow[2];
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const float l = osum[2 * ri];
    lrow[ri] = (l > 0.f && qr[ri] < n_live) ? 1.f / l : 0.f;
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
