// C ABI of shrimp_b200 (declared in include/shrimp_b200.h): argument checks,
// workspace layout, kernel launches and the ShrimpNet serve-forward schedule.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>

#include "../../include/shrimp_b200.h"
#include "attention.cuh"
#include "attention_geo.cuh"
#include "aux.cuh"
#include "gemm.cuh"
#include "conv_ts.cuh"
#include "conv_grid.cuh"
#include "mlp.cuh"

namespace sb {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

// SHRIMP_B200_SYNC_DEBUG=1: synchronise and log after every launch (debugging
// aid; never set in serving).
bool sync_debug() {
  static const bool v = [] {  // read once (thread-safe static initialisation)
    const char* e = getenv("SHRIMP_B200_SYNC_DEBUG");
    return e && e[0] == '1';
  }();
  return v;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && sync_debug()) {
    fprintf(stderr, "[sb] launched %s ...", what);
    fflush(stderr);
    e = cudaDeviceSynchronize();
    fprintf(stderr, " done (%s)\n", cudaGetErrorString(e));
  }
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return SB_OK;
}

inline long long cdiv(long long a, long long b) { return (a + b - 1) / b; }

// Programmatic dependent launch inside the forward: every kernel after the
// first is launched with the programmatic-serialization attribute, so its
// CTAs start their prologue (barriers, TMEM, tensor-map prefetch, constant
// loads, the first weight tiles) while the previous kernel drains; each kernel
// waits (griddepcontrol) before it touches activations. Measured on B200
// under CUDA-graph replay (main-size net, p50): batch 256 -2.7 %, 384 -6.7 %,
// 512 -6.2 %, 768 -3.0 %, 1024 -1.5 %, but +6 % at batch 16-64 and +0.6-0.8 %
// at 2048-4096. So it is on for 256 <= B <= 1024. SHRIMP_B200_PDL=0 / =1
// forces it off / on for every batch.
constexpr int kPdlMinBatch = 256;
constexpr int kPdlMaxBatch = 1024;
int pdl_setting() {  // -1 automatic, 0 off, 1 on; read once
  static const int v = [] {
    const char* e = getenv("SHRIMP_B200_PDL");
    return (e && strcmp(e, "1") == 0) ? 1 : (e && strcmp(e, "0") == 0) ? 0 : -1;
  }();
  return v;
}
bool pdl_for_batch(int B) {
  const int v = pdl_setting();
  return v < 0 ? (B >= kPdlMinBatch && B <= kPdlMaxBatch) : v == 1;
}
static thread_local bool t_pdl = false;  // set while the forward schedule is being issued
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(t_pdl) { t_pdl = on; }
  ~PdlScope() { t_pdl = prev; }
};

template <typename... KArgs, typename... Args>
void launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = t_pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);  // errors surface in check_launch
}
inline int round_up(int a, int b) { return (a + b - 1) / b * b; }

// N tile for an n-wide GEMM: one tile when n <= 256, else the fewest equal
// tiles (multiples of 16) of at most 256 columns.
int choose_bn(int n) {
  if (n % 32 != 0) return -1;
  for (int k = 1; k <= 32; ++k) {
    if (n % k) continue;
    const int bn = n / k;
    if (bn <= 256 && bn % 32 == 0) return bn;
  }
  return -1;
}

// Raise a kernel's dynamic shared-memory limit once per (device, kernel).
int ensure_smem(const void* fn, int bytes) {
  struct Entry { const void* fn; int dev; int bytes; };
  static thread_local Entry cache[64];
  static thread_local int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev && cache[i].bytes >= bytes) return SB_OK;
  const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, "shared-memory attribute: %s", cudaGetErrorString(e));
  if (used < 64) cache[used++] = Entry{fn, dev, bytes};
  return SB_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  // looked up until found; host threads racing on the first lookup store the same pointer
  static std::atomic<EncodeTiledFn> cached{nullptr};
  EncodeTiledFn fn = cached.load(std::memory_order_acquire);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
      cached.store(fn, std::memory_order_release);
    }
  }
  return fn;
}

// 2D row-major 16-bit tensor map, 128-byte swizzle, box {64 columns, box_rows}.
int make_tmap(CUtensorMap* m, const void* ptr, bool bf16, long long cols, long long rows, long long row_elems,
              int box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_elems * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SB_OK;
}

// 2D row-major tensor map with an explicit element type, box and swizzle
// (epilogue stores / residual loads of the TMA epilogue).
int make_tmap_ex(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int esize, long long cols, long long rows,
                 long long row_elems, int box_cols, int box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_elems * esize};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled (epilogue) failed (%d)", (int)r);
  return SB_OK;
}

// 3D map (columns, rows of a block, blocks) over a row-major buffer whose
// blocks of `rows` rows follow each other; box {32 columns, 32 rows, 1 block}.
int make_tmap_3d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int esize, long long cols, long long rows,
                 long long blocks, long long row_elems, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)blocks};
  cuuint64_t strides[2] = {(cuuint64_t)row_elems * esize, (cuuint64_t)(row_elems * rows) * esize};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = fn(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled (3D) failed (%d)", (int)r);
  return SB_OK;
}

int num_sms() {
  // per device; host threads racing on a first query store the same value
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (!n) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename T>
int launch_gemm(GemmArgs a, cudaStream_t st) {
  if (a.M <= 0) return SB_OK;
  if (a.bn <= 0) a.bn = choose_bn(a.n_total);
  if (a.bn <= 0 || a.bn > 256 || a.bn % 32 || a.n_total % a.bn)
    return fail(SB_ERR_UNSUPPORTED, "gemm: N=%d cannot be tiled (need a multiple of 32)", a.n_total);
  if (a.kpad % kChunkK || a.kpad < a.taps * a.cin)
    return fail(SB_ERR_INVALID_ARG, "gemm: kpad=%d must be a multiple of 64 covering taps*cin=%d", a.kpad,
                a.taps * a.cin);
  if (a.cin % 8) return fail(SB_ERR_UNSUPPORTED, "gemm: input channels per tap (%d) must be a multiple of 8", a.cin);
  if (a.taps < 1 || a.taps > kMaxTaps) return fail(SB_ERR_UNSUPPORTED, "gemm: %d taps > %d", a.taps, kMaxTaps);
  if (!a.gidx && a.taps != 1) return fail(SB_ERR_INVALID_ARG, "gemm: identity rows need taps == 1");
  if ((a.flags & (EPI_LN_A | EPI_LN_B | EPI_HEAD | EPI_RESID)) && a.bn != a.n_total)
    return fail(SB_ERR_UNSUPPORTED, "gemm: row-wise epilogue needs N=%d <= 256", a.n_total);
  if (a.n_total > 1024) return fail(SB_ERR_UNSUPPORTED, "gemm: N=%d > 1024", a.n_total);
  if (a.a_rows <= 0) a.a_rows = a.gidx ? (1LL << 31) - 1 : a.M;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap ma, mb;
  memset(&ma, 0, sizeof(ma));
  memset(&mb, 0, sizeof(mb));
  a.use_tma = (a.cin % kChunkK == 0) && (a.lda % 8 == 0) && ((uintptr_t)a.A % 16 == 0) &&
              ((uintptr_t)a.Bw % 16 == 0) && a.a_rows < (1LL << 31) - 1;
  if (a.use_tma) {
    if (int s = make_tmap(&ma, a.A, bf16, a.lda, a.a_rows, a.lda, a.gidx ? 1 : kBlockM)) return s;
    if (int s = make_tmap(&mb, a.Bw, bf16, a.kpad, a.n_total, a.kpad, a.bn)) return s;
  }
  // TMA epilogue: identity rows (output row = GEMM row), whole 32-column
  // chunks per half tile, no per-row head / 16-bit residual.
  CUtensorMap m16, m32, m32b;
  memset(&m16, 0, sizeof(m16));
  memset(&m32, 0, sizeof(m32));
  memset(&m32b, 0, sizeof(m32b));
  // gathered rows qualify when their outputs run contiguously in whole
  // 32-row quadrants (position blocks of a multiple of 32 rows)
  const bool rows_contig =
      !a.gidx || (a.orow_from_gidx && a.orow_run > 0 && a.orow_run % 32 == 0 && a.M % 32 == 0);
  a.tma_epi = a.use_tma && rows_contig && (a.bn / 2) % 32 == 0 && !(a.flags & (EPI_HEAD | EPI_RES16)) &&
              ((uintptr_t)a.out16 % 16 == 0) && ((uintptr_t)a.out32 % 16 == 0) && ((uintptr_t)a.out32b % 16 == 0) &&
              (a.ld16 * 2) % 16 == 0 && (a.ld32 * 4) % 16 == 0 && (a.ld32b * 4) % 16 == 0;
  if (a.tma_epi) {
    const CUtensorMapDataType dt16 = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const long long orows = a.gidx ? a.a_rows : a.M;  // gathered: outputs share the input's row layout
    if (a.flags & EPI_OUT16)
      if (int s = make_tmap_ex(&m16, a.out16, dt16, 2, a.n_total, orows, a.ld16, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return s;
    if (a.flags & (EPI_OUT32 | EPI_RESID))
      if (int s = make_tmap_ex(&m32, a.out32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.n_total, orows, a.ld32, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_128B))
        return s;
    if (a.flags & EPI_OUT32B)
      if (int s = make_tmap_ex(&m32b, a.out32b, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.n_total, orows, a.ld32b, 32,
                               32, CU_TENSOR_MAP_SWIZZLE_128B))
        return s;
  }
  const int stages = gemm_stages(a.bn, a.taps, a.tma_epi);
  const int smem = gemm_smem_bytes(a.bn, stages, a.taps, a.tma_epi);
  const bool heavy = (a.flags & (EPI_RESID | EPI_RES16 | EPI_LN_B)) != 0;
  const int variant = (heavy ? 1 : 0) + (a.tma_epi ? 2 : 0);
  const void* fns[4] = {reinterpret_cast<const void*>(gemm_ws_kernel<T, false, false>),
                        reinterpret_cast<const void*>(gemm_ws_kernel<T, true, false>),
                        reinterpret_cast<const void*>(gemm_ws_kernel<T, false, true>),
                        reinterpret_cast<const void*>(gemm_ws_kernel<T, true, true>)};
  if (int s = ensure_smem(fns[variant], smem)) return s;
  const long long tiles = cdiv(a.M, kBlockM) * (a.n_total / a.bn);
  const int grid = (int)(tiles < num_sms() ? tiles : num_sms());
  switch (variant) {
    case 0: launch_ex(gemm_ws_kernel<T, false, false>, grid, kGemmThreads, smem, st, a, ma, mb, m16, m32, m32b, stages); break;
    case 1: launch_ex(gemm_ws_kernel<T, true, false>, grid, kGemmThreads, smem, st, a, ma, mb, m16, m32, m32b, stages); break;
    case 2: launch_ex(gemm_ws_kernel<T, false, true>, grid, kGemmThreads, smem, st, a, ma, mb, m16, m32, m32b, stages); break;
    default: launch_ex(gemm_ws_kernel<T, true, true>, grid, kGemmThreads, smem, st, a, ma, mb, m16, m32, m32b, stages);
  }
  if (sync_debug())
    fprintf(stderr, "[sb] gemm M=%d N=%d bn=%d kpad=%d taps=%d cin=%d tma=%d tma_epi=%d stages=%d smem=%d grid=%d "
            "flags=%d\n", a.M, a.n_total, a.bn, a.kpad, a.taps, a.cin, a.use_tma, a.tma_epi, stages, smem, grid, a.flags);
  return check_launch("gemm_ws_kernel");
}

// Fused attention-block MLP (mlp_kernel) for C = 64 or 128; returns 1 for
// other widths (the caller then runs fc1 and fc2 as two GEMMs), else an
// sb_status (operands must be 16-byte aligned). w1: [2C][C] and w2: [C][2C]
// packed K-major 16-bit weights; out32: the fp32 stream (residual, updated in
// place); out16: the LayerNorm'd 16-bit rows.
inline bool mlp_fused_width(int C) { return C == 64 || C == 128; }
template <typename T>
int launch_mlp(const MlpArgs& a, const void* w1, const void* w2, float* out32, void* out16, cudaStream_t st) {
  if (a.M <= 0) return SB_OK;
  const int C = a.C;
  if (!mlp_fused_width(C)) return 1;
  if ((uintptr_t)a.X % 16 || (uintptr_t)w1 % 16 || (uintptr_t)w2 % 16 || (uintptr_t)out32 % 16 ||
      (uintptr_t)out16 % 16)
    return fail(SB_ERR_INVALID_ARG, "mlp: operands must be 16-byte aligned");
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mx, m1, m2, m16, m32;
  if (int s = make_tmap(&mx, a.X, bf16, C, a.M, C, kBlockM)) return s;
  if (int s = make_tmap(&m1, w1, bf16, C, 2 * C, C, 2 * C)) return s;
  if (int s = make_tmap(&m2, w2, bf16, 2 * C, C, 2 * C, C)) return s;
  const CUtensorMapDataType dt16 = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (int s = make_tmap_ex(&m16, out16, dt16, 2, C, a.M, C, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) return s;
  if (int s = make_tmap_ex(&m32, out32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, C, a.M, C, 32, 32,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return s;
  const int smem = mlp_smem_bytes(C);
  if (int s = ensure_smem(reinterpret_cast<const void*>(mlp_kernel<T>), smem)) return s;
  const long long tiles = cdiv(a.M, kBlockM);
  const int grid = (int)(tiles < num_sms() ? tiles : num_sms());
  launch_ex(mlp_kernel<T>, grid, kMlpThreads, smem, st, a, mx, m1, m2, m16, m32, out32);
  return check_launch("mlp_kernel");
}

// Position-windowed 7-tap conv (conv_ts_kernel) when the shape allows it:
// C = Cin = Cout in {64, 128, 192}, whole positions of <= 128 cells
// per 128-row tile, a window of <= 256 X rows. Returns 1 when not eligible
// (the caller then runs the gather-GEMM), else an sb_status.
template <typename T>
int launch_conv_ts(GemmArgs a, int npos, int cells, int xrows, cudaStream_t st) {
  const int C = a.n_total;
  // Input channels: C (64-column boxes), or a narrow 16 / 32 (the stem's
  // feature planes: one box of cin columns, K chunks spanning several taps).
  const bool narrow = a.cin == 16 || a.cin == 32;
  // TMEM: two C-column accumulators plus >= 2 A slots of 32 columns in 512.
  // taps: the 7-tap hex conv, or the 19-tap ray conv (16-bit residual epilogue only)
  if ((a.taps != 7 && a.taps != 19) || !a.gidx || (a.cin != C && !narrow) || C % 64 || 2 * C + 64 > 512 ||
      cells <= 0 || cells > kBlockM || xrows < cells)
    return 1;
  if (a.taps == 19 && (narrow || a.flags != (EPI_RES16 | EPI_OUT16))) return 1;
  if (a.lda != a.cin || (uintptr_t)a.A % 16 || (uintptr_t)a.Bw % 16) return 1;
  // positions per tile: 4, 2 or 1 (each position owns 128 / ppt TMEM lanes)
  int ppt = 4;
  while (ppt > 1 && (cells > kBlockM / ppt || ppt * xrows > 256)) ppt >>= 1;
  if (cells > kBlockM / ppt || ppt * xrows > 256) return 1;
  const int win_rows = ppt * xrows;
  // Rows written by TMA (fp32 outputs, residual loads) use the TMA epilogue. A
  // 16-bit-only output takes it too when the tiles fill more than one wave;
  // in a single wave (MCTS-size batches) the light instantiation, with its
  // second builder set and per-row stores, has the shorter per-tile latency
  // (B200, main shape: 15.4 vs 18.2 us per conv at B=256; 125 vs 128 us at
  // B=4096 the other way round).
  const long long conv_tiles = (npos + ppt - 1) / ppt;
  const bool heavy = (a.flags & (EPI_RESID | EPI_RES16 | EPI_LN_B | EPI_OUT32)) != 0 ||
                     ((a.flags & EPI_OUT16) != 0 && conv_tiles > num_sms());
  if (heavy && (a.flags & (EPI_OUT32B | EPI_HEAD))) return 1;  // not in the TMA epilogue
  // the 16-bit residual comes through the fp32 map's slot: not both
  if ((a.flags & EPI_RES16) && (a.flags & (EPI_RESID | EPI_OUT32 | EPI_LN_B))) return 1;
  const int stages = conv_ts_stages(C, win_rows, heavy);
  const int smem = conv_ts_smem_bytes(C, stages, win_rows, heavy);
  if (smem > 227 * 1024) return 1;
  if (a.M <= 0 || npos <= 0) return SB_OK;
  a.bn = C;
  a.kpad = round_up(a.taps * a.cin, kChunkK);
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mx, mw;
  memset(&mx, 0, sizeof(mx));
  memset(&mw, 0, sizeof(mw));
  if (narrow) {
    if (int s = make_tmap_ex(&mx, a.A, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                             a.cin, (long long)npos * xrows, a.cin, a.cin, win_rows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return s;
  } else if (int s = make_tmap(&mx, a.A, bf16, C, (long long)npos * xrows, C, win_rows)) {
    return s;
  }
  if (int s = make_tmap(&mw, a.Bw, bf16, a.kpad, C, a.kpad, C)) return s;
  // heavy epilogue: TMA stores / residual loads through 3D maps (columns,
  // rows of a position's block, positions): rows past a block are clipped
  CUtensorMap m16, m32;
  memset(&m16, 0, sizeof(m16));
  memset(&m32, 0, sizeof(m32));
  if (heavy) {
    if ((uintptr_t)a.out16 % 16 || (uintptr_t)a.out32 % 16 || (a.ld16 * 2) % 16 || (a.ld32 * 4) % 16) return 1;
    const CUtensorMapDataType dt16 = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (a.flags & EPI_OUT16)
      if (int s = make_tmap_3d(&m16, a.out16, dt16, 2, C, xrows, npos, a.ld16, CU_TENSOR_MAP_SWIZZLE_64B)) return s;
    if (a.flags & EPI_RES16) {
      // 16-bit residual rows, staged like the 16-bit outputs
      if ((uintptr_t)a.res16 % 16 || (a.ldr16 * 2) % 16) return 1;
      if (int s = make_tmap_3d(&m32, a.res16, dt16, 2, C, xrows, npos, a.ldr16, CU_TENSOR_MAP_SWIZZLE_64B)) return s;
    } else if (int s = make_tmap_3d(&m32, a.out32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, C, xrows, npos, a.ld32,
                                    CU_TENSOR_MAP_SWIZZLE_128B)) {
      return s;
    }
  }
  const bool ray = a.taps == 19;
  if (ray && !heavy) return 1;
  const void* fn = ray     ? reinterpret_cast<const void*>(conv_ts_kernel<T, true, 19>)
                   : heavy ? reinterpret_cast<const void*>(conv_ts_kernel<T, true>)
                           : reinterpret_cast<const void*>(conv_ts_kernel<T, false>);
  if (int s = ensure_smem(fn, smem)) return s;
  ConvTsGeom geo{ppt, cells, xrows, npos, xrows - cells};
  const int tiles = (npos + ppt - 1) / ppt;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  if (ray)
    launch_ex(conv_ts_kernel<T, true, 19>, grid, conv_ts_threads(true), smem, st, a, geo, mx, mw, m16, m32, stages);
  else if (heavy)
    launch_ex(conv_ts_kernel<T, true>, grid, conv_ts_threads(true), smem, st, a, geo, mx, mw, m16, m32, stages);
  else
    launch_ex(conv_ts_kernel<T, false>, grid, conv_ts_threads(false), smem, st, a, geo, mx, mw, m16, m32, stages);
  if (sync_debug())
    fprintf(stderr, "[sb] conv_ts M=%d C=%d ppt=%d win=%d stages=%d smem=%d grid=%d flags=%d\n", a.M, C, ppt,
            win_rows, stages, smem, grid, a.flags);
  return check_launch("conv_ts_kernel");
}

// The grid conv (conv_grid_kernel) for the forward's 7-tap convs with C = Cin
// = Cout a multiple of 64 (<= 128). `geo.slot_cell` comes from
// grid_geom_kernel; the kernel returns at once unless *flag == 1. Returns 1
// when the shape is not eligible.
template <typename T>
int launch_conv_grid(GemmArgs a, const GridGeom& geo, const int* flag, int skip_value, cudaStream_t st) {
  const int C = a.n_total;
  if (a.taps != 7 || !a.gidx || a.cin != C || C % 64 || C > 128 || geo.npad > kGridMaxCells) return 1;
  if (a.lda != a.cin || (uintptr_t)a.A % 16 || (uintptr_t)a.Bw % 16) return 1;
  // Residual convs keep the windowed kernel: its TMA epilogue moves the fp32
  // stream rows in bulk, where this kernel's slot-ordered rows would need one
  // scattered row access per thread.
  if (a.flags & (EPI_RES16 | EPI_OUT32B | EPI_RESID | EPI_LN_B)) return 1;
  if (geo.npos <= 0) return SB_OK;
  a.bn = C;
  a.kpad = round_up(7 * a.cin, kChunkK);
  a.skip_flag = flag;
  a.skip_value = skip_value;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mw;
  memset(&mw, 0, sizeof(mw));
  if (int s = make_tmap(&mw, a.Bw, bf16, a.kpad, C, a.kpad, C)) return s;
  const bool heavy = (a.flags & (EPI_RESID | EPI_LN_B)) != 0;
  const int smem = conv_grid_smem_bytes(C);
  const void* fn = heavy ? reinterpret_cast<const void*>(conv_grid_kernel<T, true>)
                         : reinterpret_cast<const void*>(conv_grid_kernel<T, false>);
  if (int s = ensure_smem(fn, smem)) return s;
  const long long tiles = cdiv((long long)geo.npos * kGridBlock, kBlockM);
  const long long jobs = cdiv(tiles, 2);
  const int grid = (int)(jobs < num_sms() ? jobs : num_sms());
  if (heavy)
    launch_ex(conv_grid_kernel<T, true>, grid, kGridThreads, smem, st, a, geo, mw);
  else
    launch_ex(conv_grid_kernel<T, false>, grid, kGridThreads, smem, st, a, geo, mw);
  if (sync_debug())
    fprintf(stderr, "[sb] conv_grid M=%d C=%d npos=%d smem=%d grid=%d flags=%d\n", a.M, C, geo.npos, smem, grid,
            a.flags);
  return check_launch("conv_grid_kernel");
}

// 7-tap conv over whole positions: the windowed kernel when eligible, else
// the gather-GEMM.
template <typename T>
int launch_conv(const GemmArgs& a, int npos, int cells, int xrows, cudaStream_t st) {
  int r = launch_conv_ts<T>(a, npos, cells, xrows, st);
  if (r != 1) return r;
  GemmArgs g = a;
  if (g.orow_from_gidx) g.orow_run = cells;  // each position's cells are consecutive output rows
  return launch_gemm<T>(g, st);
}

template <typename T>
int launch_attention(AttnArgs a, cudaStream_t st) {
  if (a.D % 8 || a.D <= 0 || a.D > 64)
    return fail(SB_ERR_UNSUPPORTED, "attention: head_dim=%d must be a multiple of 8 in [8, 64]", a.D);
  if (a.table_rows <= 0 || a.table_rows > kMaxTableRows)
    return fail(SB_ERR_UNSUPPORTED, "attention: %d bias rows (1..%d supported)", a.table_rows, kMaxTableRows);
  const int dp = round_up(a.D, 16);
  // Geometry-cached kernel: head_dim 16, whole 64-column boxes of heads,
  // q | k | v as the column blocks of one row-major buffer.
  if (a.mode == BIAS_COORDS && !a.own_geometry && !a.seq_lens && a.D == kGeoD && a.H % 4 == 0 && a.S > a.ntok &&
      a.S <= kGeoMaxS && 2 * (a.S - a.ntok) + a.S <= kGeoThreads && a.table_rows <= 255 && a.coords && a.lut) {
    const long long C = (long long)a.H * a.D;
    const T* q = reinterpret_cast<const T*>(a.q);
    const AttnGeoLayout L = attn_geo_layout(a.S);
    if (a.k == q + C && a.v == q + 2 * C && a.row_stride == 3 * C && a.head_stride == a.D &&
        a.pos_stride == (long long)a.S * 3 * C && (uintptr_t)a.q % 16 == 0 && L.total <= 227 * 1024 &&
        L.nj >= 8 && L.nj <= 10) {
      if (a.B <= 0) return SB_OK;
      CUtensorMap tm;
      memset(&tm, 0, sizeof(tm));
      if (int s = make_tmap(&tm, a.q, std::is_same<T, __nv_bfloat16>::value, 3 * C, (long long)a.B * a.S, 3 * C,
                            a.S))
        return s;
      // two CTAs per SM, each on one group of four heads; a group's CTAs
      // stride over the positions
      const int groups = a.H / kGeoHeads;
      const int per_group = a.B < 2 * num_sms() / groups ? a.B : 2 * num_sms() / groups;
      const int grid = groups * (per_group > 0 ? per_group : 1);
#define SB_GEO_CASE(NJV)                                                                              \
  case NJV:                                                                                           \
    if (int s = ensure_smem(reinterpret_cast<const void*>(attn_geo_kernel<T, NJV>), L.total)) return s; \
    launch_ex(attn_geo_kernel<T, NJV>, (unsigned)grid, kGeoThreads, L.total, st, a, tm);              \
    return check_launch("attn_geo_kernel");
      switch (L.nj) {
        SB_GEO_CASE(8)
        SB_GEO_CASE(9)
        SB_GEO_CASE(10)
        default: break;
      }
#undef SB_GEO_CASE
    }
  }
  // Position-resident kernel when the per-position row table and the K/V of at
  // least one head fit in shared memory: the largest head group that allows
  // two CTAs per SM, else one CTA per SM. Longer sequences stream.
  int group = 0;
  if (a.table_rows <= 255 || a.mode == BIAS_OFFSET) {
    for (int budget : {113 * 1024, 227 * 1024}) {
      for (int gsz = a.H; gsz >= 1 && !group; --gsz)
        if (attn_smem_bytes(a.S, dp, gsz, a.table_rows) <= budget) group = gsz;
      if (group) break;
    }
  }
  // The resident kernel runs one CTA per position. When the batch leaves SM
  // slots empty and the keys take more than one softmax step, the streaming
  // kernel's (query block, head, position) grid finishes sooner: this is the
  // case of the small, long-sequence groups of an evaluator payload.
  if (group && a.mode == BIAS_COORDS && attn_pad16(a.S) > 80) {
    const int per_sm = attn_smem_bytes(a.S, dp, group, a.table_rows) <= 113 * 1024 ? 2 : 1;
    if (a.B < per_sm * num_sms()) group = 0;
  }
  if (group) {
    a.group = group;
    const int smem = attn_smem_bytes(a.S, dp, group, a.table_rows);
    const int per_sm = smem <= 113 * 1024 ? 2 : 1;
    const int grid = a.B < per_sm * num_sms() ? a.B : per_sm * num_sms();
    const bool one_pass = attn_pad16(a.S) <= 80;  // all keys in one softmax step
#define SB_ATTN_CASE(DPV)                                                                       \
  case DPV: {                                                                                   \
    const void* fn = one_pass ? reinterpret_cast<const void*>(attn_kernel<T, DPV, 10>)          \
                              : reinterpret_cast<const void*>(attn_kernel<T, DPV, 4>);          \
    if (int s = ensure_smem(fn, smem)) return s;                                                \
    if (one_pass)                                                                               \
      launch_ex(attn_kernel<T, DPV, 10>, (unsigned)grid, kAttnThreads, smem, st, a);            \
    else                                                                                        \
      launch_ex(attn_kernel<T, DPV, 4>, (unsigned)grid, kAttnThreads, smem, st, a);             \
    return check_launch("attn_kernel");                                                         \
  }
    switch (dp) {
      SB_ATTN_CASE(16)
      SB_ATTN_CASE(32)
      SB_ATTN_CASE(48)
      SB_ATTN_CASE(64)
      default: break;
    }
#undef SB_ATTN_CASE
    return fail(SB_ERR_UNSUPPORTED, "attention: head_dim=%d", a.D);
  }
  dim3 grid((unsigned)cdiv(a.S, kStreamBlockQ), (unsigned)a.H, (unsigned)a.B);
#define SB_ATTN_CASE(DPV)                                                                   \
  case DPV: {                                                                               \
    const int smem = AttnStreamSmem<DPV>::kBytes;                                           \
    if (int s = ensure_smem(reinterpret_cast<const void*>(attn_stream_kernel<T, DPV>), smem)) return s; \
    launch_ex(attn_stream_kernel<T, DPV>, grid, kStreamThreads, smem, st, a);              \
    return check_launch("attn_stream_kernel");                                              \
  }
  switch (dp) {
    SB_ATTN_CASE(16)
    SB_ATTN_CASE(32)
    SB_ATTN_CASE(48)
    SB_ATTN_CASE(64)
    default: break;
  }
#undef SB_ATTN_CASE
  return fail(SB_ERR_UNSUPPORTED, "attention: head_dim=%d", a.D);
}

// ---- forward workspace --------------------------------------------------------

// Readable bytes kept after every gather table (the GEMM prefetches it in
// whole 16-byte pieces).
constexpr size_t kGidxSlack = 64;

// Workspace of the hex_conv entry points for `rows` = batch * npad cells: the
// absolute gather table (7 int32 per row, plus the prefetch slack, rounded to
// 256 bytes) followed by the fp32 row mask.
constexpr size_t hex_conv_workspace_for(size_t rows) {
  return ((rows * 7 * 4 + kGidxSlack + 255) & ~size_t(255)) + rows * 4;
}

struct FwdLayout {
  size_t seq32, xa16, y16, qkv16, o16, u16, feat16, gidx, rowmask, coords32, seqlen, slotcell, gflag;
  size_t pol32, vlog, mllog;  // payload path only: policy and head logits of a group
  size_t pool, poolc;         // cell-mean unit sums (pool_cells_apart batches only)
  size_t total;
};

// Batches whose heads_kernel grid (four positions per CTA) is less than one
// CTA per SM, with more than one pooling chunk of cells, pool the cell mean
// in pool_cells_kernel first: one warp per (position, chunk, parity) unit.
bool pool_cells_apart(int B, int npad) { return cdiv(B, 4) < num_sms() && pool_chunks(npad) > 1; }

FwdLayout fwd_layout(int C, int B, int npad, bool payload) {
  const size_t S = (size_t)npad + kNumTok;
  const size_t R = (size_t)B * S;
  const size_t Mc = (size_t)B * npad;
  FwdLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  L.seq32 = take(R * C * 4);
  L.xa16 = take(R * C * 2);
  L.y16 = take(R * C * 2);
  L.qkv16 = take(R * 3 * C * 2);
  L.o16 = take(R * C * 2);
  // the MLP hidden rows: only the unfused fc1 -> fc2 path (C not 64 / 128) keeps them in HBM
  L.u16 = take(mlp_fused_width(C) ? 0 : R * 2 * C * 2);
  L.feat16 = take(R * kFeatPad * 2);
  L.gidx = take(Mc * 7 * 4 + kGidxSlack);
  L.rowmask = take(R * 4);
  L.coords32 = take(Mc * 2 * 4);
  L.seqlen = take((size_t)B * 4);
  L.slotcell = take((size_t)B * kGridBlock * 2);
  L.gflag = take(4);
  if (payload) {
    L.pol32 = take(Mc * 4);
    L.vlog = take((size_t)B * kBins * 4);
    L.mllog = take((size_t)B * kBins * 4);
  }
  if (pool_cells_apart(B, npad)) {
    const size_t units = (size_t)B * pool_chunks(npad) * 2;
    L.pool = take(units * C * 4);
    L.poolc = take(units * 4);
  }
  L.total = off;
  return L;
}

int validate_net(const sb_net* net) {
  if (!net) return fail(SB_ERR_INVALID_ARG, "net is NULL");
  const int C = net->channels, H = net->heads;
  if (C <= 0 || C > 256 || C % 32) return fail(SB_ERR_UNSUPPORTED, "channels=%d: need a multiple of 32 <= 256", C);
  if (H <= 0 || C % H) return fail(SB_ERR_INVALID_ARG, "channels=%d not divisible by heads=%d", C, H);
  const int D = C / H;
  if (D % 8 || D > 64) return fail(SB_ERR_UNSUPPORTED, "head_dim=%d: need a multiple of 8 <= 64", D);
  const int nb = net->num_blocks;
  if (nb <= 0 || nb > SB_MAX_BLOCKS || (int)strnlen(net->layout, SB_MAX_BLOCKS + 1) != nb)
    return fail(SB_ERR_INVALID_ARG, "layout length %d invalid", nb);
  if (net->layout[nb - 1] != 'A') return fail(SB_ERR_INVALID_ARG, "layout must end with 'A'");
  for (int i = 0; i < nb; ++i)
    if (net->layout[i] != 'A' && net->layout[i] != 'C') return fail(SB_ERR_INVALID_ARG, "layout char %d", i);
  return SB_OK;
}

// Output and input bindings of one forward over B positions of npad cells.
struct FwdIo {
  const PrepArgs* dense;      // the module's (B, Npad, ...) tensors, or
  const PrepCsrArgs* csr;     // rows [row0, row0 + B) of a serve payload
  float* policy;              // (B, npad) logits
  float* value_logits;        // (B, 65)
  float* value;               // (B) decoded, or NULL
  float* ml_logits;           // (B, 65), or NULL (moves-left not requested)
  float* ml;                  // (B) decoded, or NULL
  const int32_t* legal;       // reply priors (payload path): legal-prefix lengths,
  const int64_t* prior_offs;  //   flat offsets,
  float* priors;              //   flat priors (NULL: no reply priors),
  float* priors_logits;       //   flat raw logits or NULL
  int* err;
};

// The serve forward (model.py:972-1003) over one workspace: input staging,
// stem, the trunk layout, policy conv + head, value / moves-left heads.
int forward_body(const sb_net* net, int B, int npad, const FwdLayout& L, uint8_t* ws, const FwdIo& io,
                 cudaStream_t st) {
  const int C = net->channels, H = net->heads;
  float* seq32 = reinterpret_cast<float*>(ws + L.seq32);
  __half* xa16 = reinterpret_cast<__half*>(ws + L.xa16);
  __half* y16 = reinterpret_cast<__half*>(ws + L.y16);
  __half* qkv16 = reinterpret_cast<__half*>(ws + L.qkv16);
  __half* o16 = reinterpret_cast<__half*>(ws + L.o16);
  __half* u16 = reinterpret_cast<__half*>(ws + L.u16);
  __half* feat16 = reinterpret_cast<__half*>(ws + L.feat16);
  int32_t* gidx = reinterpret_cast<int32_t*>(ws + L.gidx);
  float* rowmask = reinterpret_cast<float*>(ws + L.rowmask);
  int32_t* coords32 = reinterpret_cast<int32_t*>(ws + L.coords32);
  int32_t* seqlen = reinterpret_cast<int32_t*>(ws + L.seqlen);
  int16_t* slotcell = reinterpret_cast<int16_t*>(ws + L.slotcell);
  int* gflag = reinterpret_cast<int*>(ws + L.gflag);
  int* err = io.err;
  // Batches that may lie on the radius-4 grid (the module's dense inputs with
  // at most 81 cells, C a multiple of 64 up to 128, enough positions for the
  // grid conv to repay its extra launches) get the grid conv, chosen on the
  // device by grid_geom_kernel's flag; the windowed conv is launched beside it
  // for the other outcome.
  const bool grid_ok = !io.csr && npad <= kGridMaxCells && C % 64 == 0 && C <= 128 && B >= kGridMinBatch;

  const int S = npad + kNumTok;
  const long long R = (long long)B * S;
  const long long Mc = (long long)B * npad;
  if (R > (1LL << 31) - 1) return fail(SB_ERR_UNSUPPORTED, "batch too large");
  const int D = C / H;
  const float eps = 1e-5f;

  {
    // the first kernel waits for everything before it in the stream (inputs,
    // weight packing); the ones after it chain programmatically
    const long long work = Mc > (long long)B * kNumTok ? Mc : (long long)B * kNumTok;
    if (io.csr) {
      PrepCsrArgs p = *io.csr;
      p.B = B; p.npad = npad; p.S = S;
      p.feat16 = feat16; p.gidx = gidx; p.rowmask = rowmask; p.coords32 = coords32; p.seq_lens = seqlen; p.err = err;
      prep_csr_kernel<<<(unsigned)cdiv(work, 256), 256, 0, st>>>(p);
      if (int s = check_launch("prep_csr_kernel")) return s;
    } else {
      PrepArgs p = *io.dense;
      p.B = B; p.npad = npad; p.S = S;
      p.feat16 = feat16; p.gidx = gidx; p.rowmask = rowmask; p.coords32 = coords32; p.err = err;
      p.grid_flag = grid_ok ? gflag : nullptr;
      prep_cells_kernel<<<(unsigned)cdiv(work, 256), 256, 0, st>>>(p);
      if (int s = check_launch("prep_cells_kernel")) return s;
    }
  }
  const GridGeom ggeo{B, npad, S, kNumTok, slotcell};
  PdlScope pdl_scope(pdl_for_batch(B));
  {
    const long long tot = (long long)B * kNumTok * C / 4;  // one thread per 4 channels
    launch_ex(init_tokens_kernel, (unsigned)cdiv(tot, 256), 256, 0, st, net->tokens,
              (const __half*)net->tokens_ln16, B, S, C, seq32, xa16);
    if (int s = check_launch("init_tokens_kernel")) return s;
  }
  if (grid_ok) {
    launch_ex(grid_geom_kernel, (unsigned)cdiv(B, 8), 256, 0, st, (const int32_t*)coords32, (const int32_t*)gidx,
              (const float*)rowmask, B, npad, S, slotcell, gflag);
    if (int s = check_launch("grid_geom_kernel")) return s;
  }
  // a trunk / policy conv: the grid conv and, for batches the flag rejects,
  // the windowed conv (each returns at once when the flag selects the other)
  auto conv = [&](GemmArgs g) -> int {
    if (grid_ok) {
      const int r = launch_conv_grid<__half>(g, ggeo, gflag, 0, st);
      if (r != 1) {
        if (r != SB_OK) return r;
        g.skip_flag = gflag;
        g.skip_value = 1;
      }
    }
    return launch_conv<__half>(g, B, npad, S, st);
  };

  const int nb = net->num_blocks;
  int first_attn = -1;
  for (int i = 0; i < nb; ++i)
    if (net->layout[i] == 'A') { first_attn = i; break; }
  // attention block index of the first 'A' at or after position i
  auto next_attn_index = [&](int pos) {
    int ai = 0;
    for (int i = 0; i < pos; ++i) ai += net->layout[i] == 'A';
    return ai;
  };

  auto conv_args = [&](const void* x, const void* w, const float* bias) {
    GemmArgs g{};
    g.A = x; g.lda = C; g.a_rows = R; g.cin = C; g.taps = 7; g.gidx = gidx; g.M = (int)Mc; g.orow_from_gidx = 1;
    g.Bw = w; g.kpad = round_up(7 * C, kChunkK); g.n_total = C; g.bn = C;
    g.bias = bias; g.eps = eps; g.rowmask = rowmask; g.seq_len = S; g.ntok = kNumTok; g.err = err;
    return g;
  };
  auto linear_args = [&](const void* x, int k, const void* w, int n, const float* bias) {
    GemmArgs g{};
    g.A = x; g.lda = k; g.a_rows = R; g.cin = k; g.taps = 1; g.gidx = nullptr; g.M = (int)R;
    g.Bw = w; g.kpad = round_up(k, kChunkK); g.n_total = n; g.bn = 0;
    g.bias = bias; g.eps = eps; g.rowmask = rowmask; g.seq_len = S; g.ntok = kNumTok; g.err = err;
    return g;
  };

  // stem: relu(LN(conv(feats))) * mask (model.py:865)
  {
    GemmArgs g = conv_args(feat16, net->stem_w, net->stem_b);
    g.lda = kFeatPad; g.cin = kFeatPad; g.kpad = round_up(7 * kFeatPad, kChunkK);
    g.ln_a_w = net->stem_ln_w; g.ln_a_b = net->stem_ln_b;
    g.flags = EPI_LN_A | EPI_RELU | EPI_MASK | EPI_OUT32 | EPI_OUT16;
    g.out32 = seq32; g.ld32 = C; g.out16 = xa16; g.ld16 = C;
    if (first_attn == 0) {
      g.flags |= EPI_LN_B;
      g.ln_b_w = net->attn[0].ln1_w; g.ln_b_b = net->attn[0].ln1_b;
    }
    if (int s = launch_conv<__half>(g, B, npad, S, st)) return s;
  }

  int ci = 0, ai = 0;
  for (int pos = 0; pos < nb; ++pos) {
    const bool next_is_attn = pos + 1 < nb && net->layout[pos + 1] == 'A';
    if (net->layout[pos] == 'C') {
      const sb_conv_block_weights& w = net->conv[ci++];
      GemmArgs g1 = conv_args(xa16, w.w1, w.b1);
      g1.ln_a_w = w.ln1_w; g1.ln_a_b = w.ln1_b;
      g1.flags = EPI_LN_A | EPI_RELU | EPI_MASK | EPI_OUT16;
      g1.out16 = y16; g1.ld16 = C;
      if (int s = conv(g1)) return s;
      GemmArgs g2 = conv_args(y16, w.w2, w.b2);
      g2.ln_a_w = w.ln2_w; g2.ln_a_b = w.ln2_b; g2.gamma = w.gamma;
      g2.flags = EPI_LN_A | EPI_MASK | EPI_RESID | EPI_POST_RELU | EPI_OUT32 | EPI_OUT16;
      g2.out32 = seq32; g2.ld32 = C; g2.out16 = xa16; g2.ld16 = C;
      if (next_is_attn) {
        const int na = next_attn_index(pos + 1);
        g2.flags |= EPI_LN_B;
        g2.ln_b_w = net->attn[na].ln1_w; g2.ln_b_b = net->attn[na].ln1_b;
      }
      if (int s = conv(g2)) return s;
    } else {
      const sb_attn_block_weights& w = net->attn[ai];
      // q | k | v projections of LN1(seq) (model.py:448-455)
      GemmArgs gq = linear_args(xa16, C, w.wqkv, 3 * C, w.bqkv);
      gq.flags = EPI_OUT16; gq.out16 = qkv16; gq.ld16 = 3 * C;
      if (int s = launch_gemm<__half>(gq, st)) return s;
      // biased attention core
      AttnArgs at{};
      at.q = qkv16; at.k = qkv16 + C; at.v = qkv16 + 2 * C;
      at.pos_stride = (long long)S * 3 * C; at.row_stride = 3 * C; at.head_stride = D;
      at.out = o16; at.out_pos_stride = (long long)S * C; at.out_row_stride = C; at.out_head_stride = D;
      at.B = B; at.S = S; at.H = H; at.D = D; at.ntok = kNumTok;
      at.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
      at.mode = BIAS_COORDS; at.table = w.bias_table; at.table_rows = SB_BIAS_ROWS + 1;
      at.coords = coords32; at.keymask = rowmask; at.lut = net->lut; at.err = err;
      // payload groups: live length per position (dead key / query tiles
      // skipped) and a geometry of its own per position (no shared cache)
      if (io.csr) { at.seq_lens = seqlen; at.own_geometry = 1; }
      if (int s = launch_attention<__half>(at, st)) return s;
      // out_proj, gamma * mask residual; LN2 for the MLP (model.py:511-512)
      GemmArgs go = linear_args(o16, C, w.wo, C, w.bo);
      go.flags = EPI_MASK | EPI_RESID | EPI_OUT32 | EPI_OUT16 | EPI_LN_B;
      go.gamma = w.gamma_attn; go.out32 = seq32; go.ld32 = C; go.out16 = y16; go.ld16 = C;
      go.ln_b_w = w.ln2_w; go.ln_b_b = w.ln2_b;
      if (int s = launch_gemm<__half>(go, st)) return s;
      // fc1 + GELU + fc2 + residual + LN in one kernel when C allows it
      {
        MlpArgs mp{};
        mp.X = y16; mp.M = (int)R; mp.C = C; mp.b1 = w.b1; mp.b2 = w.b2; mp.gamma = w.gamma_mlp;
        mp.rowmask = rowmask; mp.eps = eps; mp.seq_len = S; mp.ntok = kNumTok; mp.err = err;
        if (pos == nb - 1) {
          mp.ln_b_w = net->ln_final_w; mp.ln_b_b = net->ln_final_b;
        } else {
          mp.ln_b_w = net->attn[ai + 1].ln1_w; mp.ln_b_b = net->attn[ai + 1].ln1_b;
          mp.lnb_tokens = next_is_attn ? 0 : 1;
        }
        const int r = launch_mlp<__half>(mp, w.w1, w.w2, seq32, xa16, st);
        if (r != 1) {
          if (r != SB_OK) return r;
          ++ai;
          continue;
        }
      }
      // fc1 + GELU
      GemmArgs gf1 = linear_args(y16, C, w.w1, 2 * C, w.b1);
      gf1.flags = EPI_GELU | EPI_OUT16; gf1.out16 = u16; gf1.ld16 = 2 * C;
      if (int s = launch_gemm<__half>(gf1, st)) return s;
      // fc2, gamma * mask residual; LN for whatever reads the stream next
      GemmArgs gf2 = linear_args(u16, 2 * C, w.w2, C, w.b2);
      gf2.flags = EPI_MASK | EPI_RESID | EPI_OUT32 | EPI_OUT16 | EPI_LN_B;
      gf2.gamma = w.gamma_mlp; gf2.out32 = seq32; gf2.ld32 = C; gf2.out16 = xa16; gf2.ld16 = C;
      if (pos == nb - 1) {
        gf2.ln_b_w = net->ln_final_w; gf2.ln_b_b = net->ln_final_b;  // xa16 = ln_final(stream), every row
      } else {
        const int na = ai + 1;
        gf2.ln_b_w = net->attn[na].ln1_w; gf2.ln_b_b = net->attn[na].ln1_b;
        if (!next_is_attn) gf2.flags |= EPI_LNB_TOKENS;
      }
      if (int s = launch_gemm<__half>(gf2, st)) return s;
      ++ai;
    }
  }

  // policy: (relu(conv(cells)) . w + b) * mask (model.py:1011-1020)
  {
    GemmArgs g = conv_args(xa16, net->policy_conv_w, net->policy_conv_b);
    g.flags = EPI_HEAD; g.head_w = net->policy_head_w; g.head_b = net->policy_head_b; g.head_out = io.policy;
    if (int s = conv(g)) return s;
  }
  // value (+ moves-left) heads and decode (model.py:984-1003, losses.py:40-61)
  {
    HeadsArgs h{};
    h.lnf16 = xa16; h.rowmask = rowmask; h.B = B; h.S = S; h.C = C;
    h.vr_wT = net->value_red_wT; h.vr_b = net->value_red_b; h.vh_wT = net->value_head_wT; h.vh_b = net->value_head_b;
    h.value_logits = io.value_logits; h.value = io.value;
    if (io.ml_logits) {
      h.mr_wT = net->ml_red_wT; h.mr_b = net->ml_red_b; h.mh_wT = net->ml_head_wT; h.mh_b = net->ml_head_b;
      h.ml_logits = io.ml_logits; h.ml = io.ml;
    }
    if (io.priors) {
      h.policy = io.policy; h.npad = npad; h.legal = io.legal; h.prior_offs = io.prior_offs;
      h.priors = io.priors; h.priors_logits = io.priors_logits;
    }
    if (pool_cells_apart(B, npad)) {
      float* pool = reinterpret_cast<float*>(ws + L.pool);
      float* pool_cnt = reinterpret_cast<float*>(ws + L.poolc);
      const long long units = (long long)B * pool_chunks(npad) * 2;
      launch_ex(pool_cells_kernel, (unsigned)cdiv(units, kPoolThreads / 32), kPoolThreads, 0, st,
                (const __half*)xa16, (const float*)rowmask, B, S, C, pool, pool_cnt);
      if (int s = check_launch("pool_cells_kernel")) return s;
      h.pool = pool; h.pool_cnt = pool_cnt;
    }
    // positions per CTA: 4, or 8 once four per CTA would take more than
    // two waves (fewer re-reads of the layer-1 weights). Larger groups (16,
    // 32 per CTA) measured 0.2-1 % slower forwards at B=2048-4096.
    const int P = (cdiv(B, 4) > 2 * num_sms() && heads_smem_floats(C, 8) * 4 <= 113 * 1024) ? 8 : 4;
    const int smem = heads_smem_floats(C, P) * 4;
    const void* fn = P == 4 ? reinterpret_cast<const void*>(heads_kernel<4>)
                            : reinterpret_cast<const void*>(heads_kernel<8>);
    if (int s = ensure_smem(fn, smem)) return s;
    const unsigned grid = (unsigned)cdiv(B, P);
    if (P == 4)
      launch_ex(heads_kernel<4>, grid, kHeadsThreads, smem, st, h);
    else
      launch_ex(heads_kernel<8>, grid, kHeadsThreads, smem, st, h);
    if (int s = check_launch("heads_kernel")) return s;
  }
  return SB_OK;
}


}  // namespace
}  // namespace sb

using namespace sb;

extern "C" {

int sb_abi_version(void) { return SB_ABI_VERSION; }

int sb_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return SB_ERR_INVALID_ARG;
  snprintf(buf, len, "%s", g_last_error.c_str());
  return SB_OK;
}

int sb_forward_workspace_bytes(const sb_net* net, int batch, int npad, size_t* bytes) {
  if (int s = validate_net(net)) return s;
  if (!bytes || batch < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "workspace query: bad batch/npad");
  *bytes = fwd_layout(net->channels, batch, npad, false).total;
  return SB_OK;
}

int sb_forward_policy_value(const sb_net* net, const sb_inputs* in, sb_outputs* out, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (int s = validate_net(net)) return s;
  if (!in || !out || !out->policy || !out->value_logits) return fail(SB_ERR_INVALID_ARG, "inputs/outputs missing");
  const int B = in->batch, npad = in->npad;
  if (B == 0) return SB_OK;
  if (B < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "batch=%d npad=%d", B, npad);
  if (!in->feats || !in->nbr || !in->mask || !in->coords) return fail(SB_ERR_INVALID_ARG, "input pointer NULL");
  if ((long long)B * (npad + kNumTok) > (1LL << 31) - 1) return fail(SB_ERR_UNSUPPORTED, "batch too large");
  const FwdLayout L = fwd_layout(net->channels, B, npad, false);
  if (!workspace || workspace_bytes < L.total)
    return fail(SB_ERR_WORKSPACE, "workspace %zu < required %zu bytes", workspace_bytes, L.total);
  PrepArgs p{};
  p.feats = in->feats; p.feats_dtype = in->feats_dtype;
  p.nbr = in->nbr; p.nbr_dtype = in->nbr_dtype;
  p.mask = in->mask; p.mask_dtype = in->mask_dtype;
  p.coords = in->coords; p.coords_dtype = in->coords_dtype;
  FwdIo io{};
  io.dense = &p;
  io.policy = out->policy; io.value_logits = out->value_logits; io.value = out->value;
  io.ml_logits = out->ml_logits; io.ml = out->ml_logits ? out->moves_left : nullptr;
  io.err = out->status;
  return forward_body(net, B, npad, L, reinterpret_cast<uint8_t*>(workspace), io,
                      reinterpret_cast<cudaStream_t>(stream));
}

// ---- serve payload: ShrimpEvaluator.submit_payload / result ------------------

int sb_plan_groups(const int64_t* row_offsets, int batch, int quant, double waste_fraction, double pair_ceiling,
                   sb_group* groups, int* num_groups) {
  if (!row_offsets || !groups || !num_groups || batch < 0 || quant <= 0)
    return fail(SB_ERR_INVALID_ARG, "plan_groups: bad args");
  int ng = 0, start = 0;
  while (start < batch) {
    const long long first = row_offsets[start + 1] - row_offsets[start];
    const long long pad_to = first <= quant ? quant : (first + quant - 1) / quant * quant;
    const long long waste = (long long)(waste_fraction * (double)pad_to);  // truncation, as int()
    const long long floor_size = pad_to - (waste > quant ? waste : quant);
    const double s2 = (double)(pad_to + kNumTok) * (double)(pad_to + kNumTok);
    int end = start + 1;
    while (end < batch) {
      if ((double)(end - start + 1) * s2 > pair_ceiling) break;
      if (row_offsets[end + 1] - row_offsets[end] < floor_size) break;
      ++end;
    }
    for (int r = start; r < end; ++r)
      if (row_offsets[r + 1] - row_offsets[r] > pad_to || row_offsets[r + 1] < row_offsets[r])
        return fail(SB_ERR_INVALID_ARG,
                    "plan_groups: row %d has %lld nodes > the group's %lld; rows must come sorted by node count, "
                    "largest first (the payload order)", r, (long long)(row_offsets[r + 1] - row_offsets[r]), pad_to);
    if (pad_to > (1 << 20)) return fail(SB_ERR_UNSUPPORTED, "plan_groups: row of %lld nodes", first);
    groups[ng].start = start;
    groups[ng].end = end;
    groups[ng].pad_to = (int)pad_to;
    ++ng;
    start = end;
  }
  *num_groups = ng;
  return SB_OK;
}

}  // extern "C"

namespace {
// Serve groups are independent forwards: group i runs on lane i % kServeLanes,
// lane 0 being the caller's stream and lanes 1.. auxiliary streams of the
// calling host thread, each lane with its own slice of the workspace. A
// group's kernels fill only part of the GPU (hundreds of tiles), so the
// lanes overlap them. Fork and join go through events, which also works
// while the caller's stream is being captured into a CUDA graph.
constexpr int kServeLanes = 4;

struct ServeLanes {
  cudaStream_t aux[kServeLanes - 1] = {};
  cudaEvent_t fork = nullptr;
  cudaEvent_t join[kServeLanes - 1] = {};
  bool ready = false;
};

// Streams and events of this host thread on the current device (created on
// first use; driver objects, not device memory).
int serve_lanes(ServeLanes** out) {
  static thread_local ServeLanes lanes[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(SB_ERR_CUDA, "evaluate: no device");
  ServeLanes& L = lanes[dev];
  if (!L.ready) {
    for (int i = 0; i < kServeLanes - 1; ++i) {
      if (cudaStreamCreateWithFlags(&L.aux[i], cudaStreamNonBlocking) != cudaSuccess ||
          cudaEventCreateWithFlags(&L.join[i], cudaEventDisableTiming) != cudaSuccess)
        return check_launch("evaluate: lane streams");
    }
    if (cudaEventCreateWithFlags(&L.fork, cudaEventDisableTiming) != cudaSuccess)
      return check_launch("evaluate: lane events");
    L.ready = true;
  }
  *out = &L;
  return SB_OK;
}

// Workspace slice of each lane: the largest group layout among its groups.
int serve_lane_bytes(const sb_net* net, const sb_group* groups, int num_groups, size_t (&lane_bytes)[kServeLanes]) {
  for (int l = 0; l < kServeLanes; ++l) lane_bytes[l] = 0;
  for (int i = 0; i < num_groups; ++i) {
    const int g = groups[i].end - groups[i].start;
    if (g <= 0 || groups[i].pad_to <= 0) return fail(SB_ERR_INVALID_ARG, "evaluate workspace: group %d", i);
    const size_t t = (fwd_layout(net->channels, g, groups[i].pad_to, true).total + 255) & ~size_t(255);
    size_t& lb = lane_bytes[i % kServeLanes];
    lb = t > lb ? t : lb;
  }
  return SB_OK;
}
}  // namespace

extern "C" {

int sb_evaluate_workspace_bytes(const sb_net* net, const sb_group* groups, int num_groups, size_t* bytes) {
  if (int s = validate_net(net)) return s;
  if (!bytes || num_groups < 0 || (num_groups > 0 && !groups)) return fail(SB_ERR_INVALID_ARG, "evaluate workspace");
  size_t lane_bytes[kServeLanes];
  if (int s = serve_lane_bytes(net, groups, num_groups, lane_bytes)) return s;
  size_t need = 0;
  for (int l = 0; l < kServeLanes; ++l) need += lane_bytes[l];
  *bytes = need;
  return SB_OK;
}

int sb_evaluate_payload(const sb_net* net, const sb_payload* payload, const sb_group* groups, int num_groups,
                        sb_reply* reply, void* workspace, size_t workspace_bytes, void* stream) {
  if (int s = validate_net(net)) return s;
  if (!payload || !reply || num_groups < 0 || (num_groups > 0 && !groups))
    return fail(SB_ERR_INVALID_ARG, "evaluate: payload/reply/groups missing");
  if (payload->batch == 0) return SB_OK;
  if (!payload->node_feats || !payload->node_qr || !payload->nbr || !payload->row_offsets ||
      !payload->legal_counts || !payload->prior_offsets || !reply->values || !reply->priors)
    return fail(SB_ERR_INVALID_ARG, "evaluate: NULL payload or reply pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  // validate the whole plan before anything is enqueued
  int covered = 0;
  for (int i = 0; i < num_groups; ++i) {
    const sb_group& gr = groups[i];
    const int g = gr.end - gr.start;
    if (gr.start != covered || g <= 0 || gr.end > payload->batch || gr.pad_to <= 0)
      return fail(SB_ERR_INVALID_ARG, "evaluate: groups must tile rows 0..%d in order (group %d)", payload->batch, i);
    covered = gr.end;
    if ((long long)g * (gr.pad_to + kNumTok) > (1LL << 31) - 1) return fail(SB_ERR_UNSUPPORTED, "group too large");
  }
  if (covered != payload->batch) return fail(SB_ERR_INVALID_ARG, "evaluate: groups cover %d of %d rows", covered,
                                             payload->batch);
  size_t lane_bytes[kServeLanes];
  if (int s = serve_lane_bytes(net, groups, num_groups, lane_bytes)) return s;
  size_t lane_off[kServeLanes], need = 0;
  for (int l = 0; l < kServeLanes; ++l) {
    lane_off[l] = need;
    need += lane_bytes[l];
  }
  if (!workspace || workspace_bytes < need)
    return fail(SB_ERR_WORKSPACE, "evaluate: workspace %zu < required %zu bytes", workspace_bytes, need);
  const int nlanes = num_groups < kServeLanes ? num_groups : kServeLanes;
  ServeLanes* lanes = nullptr;
  cudaStream_t lane_st[kServeLanes] = {st};
  if (nlanes > 1) {
    if (int s = serve_lanes(&lanes)) return s;
    if (cudaEventRecord(lanes->fork, st) != cudaSuccess) return check_launch("evaluate: fork");
    for (int l = 1; l < nlanes; ++l) {
      lane_st[l] = lanes->aux[l - 1];
      if (cudaStreamWaitEvent(lane_st[l], lanes->fork, 0) != cudaSuccess) return check_launch("evaluate: fork wait");
    }
  }
  int status = SB_OK;
  for (int i = 0; i < num_groups && status == SB_OK; ++i) {
    const sb_group& gr = groups[i];
    const int g = gr.end - gr.start;
    const int lane = i % kServeLanes;
    uint8_t* lws = ws + lane_off[lane];
    const FwdLayout L = fwd_layout(net->channels, g, gr.pad_to, true);
    PrepCsrArgs p{};
    p.feats = payload->node_feats; p.feats_dtype = payload->feats_dtype;
    p.qr = payload->node_qr; p.nbr = payload->nbr; p.offsets = payload->row_offsets; p.row0 = gr.start;
    FwdIo io{};
    io.csr = &p;
    io.policy = reinterpret_cast<float*>(lws + L.pol32);
    io.value_logits = reinterpret_cast<float*>(lws + L.vlog);
    io.value = reply->values + gr.start;
    if (reply->moves_left) {
      io.ml_logits = reinterpret_cast<float*>(lws + L.mllog);
      io.ml = reply->moves_left + gr.start;
    }
    io.legal = payload->legal_counts + gr.start;
    io.prior_offs = payload->prior_offsets + gr.start;
    io.priors = reply->priors;
    io.priors_logits = reply->priors_logits;
    io.err = reply->status;
    status = forward_body(net, g, gr.pad_to, L, lws, io, lane_st[lane]);
  }
  // join every lane back into the caller's stream (also after an error, so a
  // capture of the caller's stream is never left with a forked stream)
  for (int l = 1; l < nlanes; ++l) {
    if (cudaEventRecord(lanes->join[l - 1], lane_st[l]) != cudaSuccess ||
        cudaStreamWaitEvent(st, lanes->join[l - 1], 0) != cudaSuccess)
      return status != SB_OK ? status : check_launch("evaluate: join");
  }
  return status;
}

int sb_build_gather_index(const void* nbr, int nbr_dtype, int batch, int npad, int32_t* out, int32_t* status,
                          void* stream) {
  if (!nbr || !out || batch < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "gather index: bad args");
  const long long n = (long long)batch * npad;
  if (n == 0) return SB_OK;
  gather_index_kernel<<<(unsigned)cdiv(n, 256), 256, 0, (cudaStream_t)stream>>>(nbr, nbr_dtype, batch, npad, out,
                                                                                 status);
  return check_launch("gather_index_kernel");
}

int sb_build_pair_u8(const void* coords, int coords_dtype, const void* mask, int mask_dtype, int batch, int npad,
                     const uint8_t* lut, uint8_t* out, void* stream) {
  if (!coords || !mask || !lut || !out || batch < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "pair: bad args");
  const long long S = npad + kNumTok;
  const long long n = (long long)batch * S * S;
  if (n == 0) return SB_OK;
  pair_u8_kernel<<<(unsigned)cdiv(n, 256), 256, 0, (cudaStream_t)stream>>>(coords, coords_dtype, mask, mask_dtype,
                                                                            batch, npad, lut, out);
  return check_launch("pair_u8_kernel");
}

// Extra workspace of the grid conv path of hex_conv (positions of at most 81
// cells): the slot table and the eligibility flag, after the base pieces.
size_t hex_conv_grid_extra(int batch, int npad) {
  return npad <= kGridMaxCells ? (((size_t)batch * kGridBlock * 2 + 255) & ~size_t(255)) + 256 : 0;
}

int sb_hex_conv_workspace_bytes(int batch, int npad, size_t* bytes) {
  if (!bytes || batch < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "hex_conv workspace: bad args");
  *bytes = hex_conv_workspace_for((size_t)batch * npad) + hex_conv_grid_extra(batch, npad);
  return SB_OK;
}

// Pieces of a hex_conv workspace (or plan) of `rows` = batch * npad rows:
// absolute gather rows, fp32 row mask and, when the grid extra is present,
// the grid slot table and the lattice flag (0 = the cells lie on the hex
// lattice, 1 = they do not).
struct HexConvTables {
  int32_t* gabs;
  float* rm;
  int16_t* slot;
  int* gflag;
};
static HexConvTables hex_conv_tables_at(void* ws, long long rows, size_t extra) {
  const size_t base_need = hex_conv_workspace_for((size_t)rows);
  HexConvTables t;
  t.gabs = reinterpret_cast<int32_t*>(ws);
  t.rm = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + ((rows * 7 * 4 + (long long)kGidxSlack + 255) & ~255LL));
  t.slot = reinterpret_cast<int16_t*>(reinterpret_cast<uint8_t*>(ws) + base_need);
  t.gflag = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ws) + base_need + extra - 256);
  return t;
}
// Batches whose tables get the grid slots (the grid conv repays its table
// only from 1024 positions of at most 81 cells on).
static bool hex_conv_grid_batch(int batch, size_t extra) { return extra > 0 && batch >= kGridMinBatch; }

// Build the tables of a gather table + mask into `ws` (grid: with the slots
// and the lattice flag, which the device sets).
static int hex_conv_build_tables(const int32_t* gather_idx, const uint8_t* mask, int batch, int npad,
                                 const HexConvTables& t, bool grid, cudaStream_t st) {
  const long long rows = (long long)batch * npad;
  if (grid) {
    // tables and grid slots in one pass; *gflag = 1 marks an ineligible batch
    if (cudaMemsetAsync(t.gflag, 0, sizeof(int), st) != cudaSuccess) return check_launch("flag reset");
    grid_embed_kernel<<<(unsigned)cdiv(batch, 8), 256, 0, st>>>(gather_idx, mask, batch, npad, t.gabs, t.rm, t.slot,
                                                                 t.gflag);
    return check_launch("grid_embed_kernel");
  }
  absolute_gidx_kernel<<<(unsigned)cdiv(rows * 7, 256), 256, 0, st>>>(gather_idx, batch, npad, 7, t.gabs);
  if (int s = check_launch("absolute_gidx_kernel")) return s;
  mask_to_float_kernel<<<(unsigned)cdiv(rows, 256), 256, 0, st>>>(mask, rows, t.rm);
  return check_launch("mask_to_float_kernel");
}

// The conv itself over built tables. grid_mode 0: windowed / gather-GEMM
// only; 1: the grid conv and the windowed conv both launched, the device flag
// choosing (each returns at once for the other outcome); 2: the caller knows
// the cells lie on the lattice: the grid conv alone when the conv shape
// allows it.
static int hex_conv_run(const void* x, const HexConvTables& t, const void* w, const float* bias, const float* ln_w,
                        const float* ln_b, float eps, int flags, int batch, int npad, int cin, int cout, void* out,
                        int grid_mode, cudaStream_t st) {
  const long long rows = (long long)batch * npad;
  GemmArgs g{};
  g.A = x; g.lda = cin; g.a_rows = rows; g.cin = cin; g.taps = 7; g.gidx = t.gabs; g.M = (int)rows;
  g.Bw = w; g.kpad = round_up(7 * cin, kChunkK); g.n_total = cout; g.bn = 0;
  g.bias = bias; g.ln_a_w = ln_w; g.ln_a_b = ln_b; g.eps = eps; g.rowmask = t.rm;
  g.flags = flags | EPI_MASK | EPI_OUT16; g.out16 = out; g.ld16 = cout;
  if (grid_mode != 0 && cin == cout && (cout == 64 || cout == 128)) {
    const GridGeom geo{batch, npad, npad, 0, t.slot};
    GemmArgs gg = g;
    const int r = launch_conv_grid<__half>(gg, geo, grid_mode == 1 ? t.gflag : nullptr, 1, st);
    if (r != 1) {
      if (r != SB_OK || grid_mode == 2) return r;
      g.skip_flag = t.gflag;
      g.skip_value = 0;
    }
  }
  return launch_conv<__half>(g, batch, npad, npad, st);
}

// allow_grid: positions of at most 81 cells whose gather table embeds in the
// hex grid run on the grid conv (the workspace then holds the slot table);
// without it only the base workspace is used.
static int hex_conv_common(const void* x, const int32_t* gather_idx, const uint8_t* mask, const void* w,
                           const float* bias, const float* ln_w, const float* ln_b, float eps, int flags,
                           int batch, int npad, int cin, int cout, void* out, void* workspace,
                           size_t workspace_bytes, void* stream, bool allow_grid) {
  if (!x || !gather_idx || !mask || !w || !bias || !out || batch < 0 || npad <= 0)
    return fail(SB_ERR_INVALID_ARG, "hex_conv: bad args");
  const size_t base_need = hex_conv_workspace_for((size_t)batch * npad);
  const size_t extra = allow_grid ? hex_conv_grid_extra(batch, npad) : 0;
  if (!workspace || workspace_bytes < base_need + extra)
    return fail(SB_ERR_WORKSPACE, "hex_conv: workspace too small");
  const long long rows = (long long)batch * npad;
  if (rows == 0) return SB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const HexConvTables t = hex_conv_tables_at(workspace, rows, extra);
  const bool grid = hex_conv_grid_batch(batch, extra) && cin == cout && (cout == 64 || cout == 128);
  if (int s = hex_conv_build_tables(gather_idx, mask, batch, npad, t, grid, st)) return s;
  return hex_conv_run(x, t, w, bias, ln_w, ln_b, eps, flags, batch, npad, cin, cout, out, grid ? 1 : 0, st);
}

int sb_hex_conv(const void* x, const int32_t* gather_idx, const uint8_t* mask, const void* w, const float* bias,
                int batch, int npad, int cin, int cout, void* out, void* workspace, size_t workspace_bytes,
                void* stream) {
  return hex_conv_common(x, gather_idx, mask, w, bias, nullptr, nullptr, 0.f, 0, batch, npad, cin, cout, out,
                         workspace, workspace_bytes, stream, true);
}

// ---- allocation-free hex_conv --------------------------------------------------
// Scratch of sb_hex_conv_noalloc: a fixed file-scope device array (absolute
// gather table + row mask), so the call needs no caller workspace and the
// library still allocates nothing at run time.
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB: up to 262,141 rows (batch * npad)
constexpr long long kNoAllocMaxRows = 262141;       // largest batch * npad whose workspace fits
static_assert(hex_conv_workspace_for(kNoAllocMaxRows) <= kNoAllocScratchBytes,
              "the documented row limit must fit the fixed scratch");
static_assert(hex_conv_workspace_for(kNoAllocMaxRows + 1) > kNoAllocScratchBytes,
              "the documented row limit must be the largest that fits");
static __device__ __align__(256) uint8_t g_hex_conv_scratch[kNoAllocScratchBytes];

int sb_hex_conv_noalloc(const void* x, const int32_t* gather_idx, const uint8_t* mask, const void* w,
                        const float* bias, int batch, int npad, int cin, int cout, void* out, void* stream) {
  if (batch < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "hex_conv_noalloc: bad args");
  const size_t need = hex_conv_workspace_for((size_t)batch * npad);  // no grid path here
  if (need > kNoAllocScratchBytes)
    return fail(SB_ERR_UNSUPPORTED,
                "hex_conv_noalloc: batch*npad=%lld rows need %zu scratch bytes; the fixed scratch holds %zu "
                "(at most %lld rows)",
                (long long)batch * npad, need, kNoAllocScratchBytes, kNoAllocMaxRows);
  // Per-device symbol address, resolved on the first call on each device
  // (that call does the set-up; later calls only read the cache). Threads
  // racing on a first call all store the same address; the entries are
  // atomic so that race is benign. The cache is not refreshed after
  // cudaDeviceReset.
  static std::atomic<void*> scratch[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(SB_ERR_CUDA, "hex_conv_noalloc: no current device");
  void* base = scratch[dev].load(std::memory_order_relaxed);
  if (!base) {
    const cudaError_t e = cudaGetSymbolAddress(&base, g_hex_conv_scratch);
    if (e != cudaSuccess || !base)
      return fail(SB_ERR_CUDA, "hex_conv_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    scratch[dev].store(base, std::memory_order_relaxed);
  }
  return hex_conv_common(x, gather_idx, mask, w, bias, nullptr, nullptr, 0.f, 0, batch, npad, cin, cout, out,
                         base, kNoAllocScratchBytes, stream, false);
}

int sb_hex_conv_ln(const void* x, const int32_t* gather_idx, const uint8_t* mask, const void* w, const float* bias,
                   const float* ln_w, const float* ln_b, float eps, int relu, int batch, int npad, int cin, int cout,
                   void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!ln_w || !ln_b) return fail(SB_ERR_INVALID_ARG, "hex_conv_ln: LayerNorm params NULL");
  return hex_conv_common(x, gather_idx, mask, w, bias, ln_w, ln_b, eps, EPI_LN_A | (relu ? EPI_RELU : 0), batch,
                         npad, cin, cout, out, workspace, workspace_bytes, stream, true);
}

// ---- planned hex_conv: the tables of one neighbour table, reused ----------
int sb_hex_conv_plan(const int32_t* gather_idx, const uint8_t* mask, int batch, int npad, void* plan,
                     size_t plan_bytes, int* lattice, void* stream) {
  if (!gather_idx || !mask || !lattice || batch < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "hex_conv_plan: bad args");
  *lattice = 0;
  const size_t extra = hex_conv_grid_extra(batch, npad);
  if (!plan || plan_bytes < hex_conv_workspace_for((size_t)batch * npad) + extra)
    return fail(SB_ERR_WORKSPACE, "hex_conv_plan: plan buffer too small");
  const long long rows = (long long)batch * npad;
  if (rows == 0) return SB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const HexConvTables t = hex_conv_tables_at(plan, rows, extra);
  const bool grid = hex_conv_grid_batch(batch, extra);
  if (int s = hex_conv_build_tables(gather_idx, mask, batch, npad, t, grid, st)) return s;
  if (grid) {
    int flag = 1;
    if (cudaMemcpyAsync(&flag, t.gflag, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return check_launch("hex_conv_plan: reading the lattice flag");
    *lattice = flag == 0 ? 1 : 0;
  }
  return SB_OK;
}

static int hex_conv_planned(const void* x, const void* plan, size_t plan_bytes, int lattice, const void* w,
                            const float* bias, const float* ln_w, const float* ln_b, float eps, int flags, int batch,
                            int npad, int cin, int cout, void* out, void* stream) {
  if (!x || !plan || !w || !bias || !out || batch < 0 || npad <= 0)
    return fail(SB_ERR_INVALID_ARG, "hex_conv_planned: bad args");
  const size_t extra = hex_conv_grid_extra(batch, npad);
  if (plan_bytes < hex_conv_workspace_for((size_t)batch * npad) + extra)
    return fail(SB_ERR_WORKSPACE, "hex_conv_planned: plan buffer too small");
  if (lattice && !hex_conv_grid_batch(batch, extra))
    return fail(SB_ERR_INVALID_ARG, "hex_conv_planned: lattice=1 for a batch the plan gave no grid slots");
  const long long rows = (long long)batch * npad;
  if (rows == 0) return SB_OK;
  const HexConvTables t = hex_conv_tables_at(const_cast<void*>(plan), rows, extra);
  return hex_conv_run(x, t, w, bias, ln_w, ln_b, eps, flags, batch, npad, cin, cout, out, lattice ? 2 : 0,
                      (cudaStream_t)stream);
}

int sb_hex_conv_planned(const void* x, const void* plan, size_t plan_bytes, int lattice, const void* w,
                        const float* bias, int batch, int npad, int cin, int cout, void* out, void* stream) {
  return hex_conv_planned(x, plan, plan_bytes, lattice, w, bias, nullptr, nullptr, 0.f, 0, batch, npad, cin, cout,
                          out, stream);
}

int sb_hex_conv_ln_planned(const void* x, const void* plan, size_t plan_bytes, int lattice, const void* w,
                           const float* bias, const float* ln_w, const float* ln_b, float eps, int relu, int batch,
                           int npad, int cin, int cout, void* out, void* stream) {
  if (!ln_w || !ln_b) return fail(SB_ERR_INVALID_ARG, "hex_conv_ln_planned: LayerNorm params NULL");
  return hex_conv_planned(x, plan, plan_bytes, lattice, w, bias, ln_w, ln_b, eps, EPI_LN_A | (relu ? EPI_RELU : 0),
                          batch, npad, cin, cout, out, stream);
}

int sb_attn_pair(const void* q, const void* k, const void* v, const uint8_t* pair, const float* table2,
                 const int32_t* seq_lens, int batch, int heads, int seq, int head_dim, void* out, void* stream) {
  if (!q || !k || !v || !pair || !table2 || !out || batch < 0 || heads <= 0 || seq <= 0)
    return fail(SB_ERR_INVALID_ARG, "attn_pair: bad args");
  if (batch == 0) return SB_OK;
  AttnArgs a{};
  a.q = q; a.k = k; a.v = v;
  a.pos_stride = (long long)heads * seq * head_dim; a.head_stride = (long long)seq * head_dim; a.row_stride = head_dim;
  a.out = out; a.out_pos_stride = a.pos_stride; a.out_head_stride = a.head_stride; a.out_row_stride = head_dim;
  a.B = batch; a.S = seq; a.H = heads; a.D = head_dim; a.ntok = 0;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  a.mode = BIAS_PAIR; a.table = table2; a.table_rows = SB_BIAS_ROWS + 1; a.pair = pair; a.seq_lens = seq_lens;
  return launch_attention<__half>(a, (cudaStream_t)stream);
}

int sb_pack_hex_conv_weight(const float* w, int taps, int cin, int cin_pad, int cout, void* out, void* stream) {
  if (!w || !out || taps <= 0 || cin <= 0 || cin_pad < cin || cout <= 0) return fail(SB_ERR_INVALID_ARG, "pack conv");
  const int kpad = round_up(taps * cin_pad, kChunkK);
  const long long n = (long long)cout * kpad;
  pack_conv_kernel<<<(unsigned)cdiv(n, 256), 256, 0, (cudaStream_t)stream>>>(w, taps, cin, cin_pad, cout, kpad,
                                                                              (__half*)out);
  return check_launch("pack_conv_kernel");
}

int sb_pack_linear_weight(const float* w, int n, int k, void* out, void* stream) {
  if (!w || !out || n <= 0 || k <= 0) return fail(SB_ERR_INVALID_ARG, "pack linear");
  const int kpad = round_up(k, kChunkK);
  const long long tot = (long long)n * kpad;
  pack_linear_kernel<<<(unsigned)cdiv(tot, 256), 256, 0, (cudaStream_t)stream>>>(w, n, k, kpad, (__half*)out);
  return check_launch("pack_linear_kernel");
}

int sb_decode_binned(const float* logits, int batch, float scale, float offset, float* out, void* stream) {
  if (!logits || !out || batch < 0) return fail(SB_ERR_INVALID_ARG, "decode: bad args");
  if (batch == 0) return SB_OK;
  decode_binned_kernel<<<(unsigned)cdiv(batch, 128), 128, 0, (cudaStream_t)stream>>>(logits, batch, scale, offset,
                                                                                      out);
  return check_launch("decode_binned_kernel");
}

int sb_legal_prefix_softmax(const float* policy, int batch, int npad, const int32_t* legal, const int64_t* offs,
                            float* out, void* stream) {
  if (!policy || !legal || !offs || !out || batch < 0 || npad <= 0) return fail(SB_ERR_INVALID_ARG, "softmax: bad args");
  if (batch == 0) return SB_OK;
  legal_softmax_kernel<<<(unsigned)cdiv((long long)batch * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      policy, batch, npad, legal, offs, out);
  return check_launch("legal_softmax_kernel");
}

int sb_raytap_conv(const void* x, const int32_t* nbr, int taps, const void* w, const float* bias, int batch, int n,
                   int c, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !nbr || !w || !bias || !out || batch < 0 || n <= 0 || taps <= 0) return fail(SB_ERR_INVALID_ARG, "raytap: bad args");
  const size_t need = (size_t)batch * n * taps * 4 + kGidxSlack;
  if (!workspace || workspace_bytes < need) return fail(SB_ERR_WORKSPACE, "raytap: workspace < %zu", need);
  if (batch == 0) return SB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  int32_t* g = reinterpret_cast<int32_t*>(workspace);
  shared_gidx_kernel<<<(unsigned)cdiv((long long)batch * n * taps, 256), 256, 0, st>>>(nbr, batch, n, taps, g);
  if (int s = check_launch("shared_gidx_kernel")) return s;
  GemmArgs a{};
  a.A = x; a.lda = c; a.a_rows = (long long)batch * n; a.cin = c; a.taps = taps; a.gidx = g; a.M = batch * n;
  a.Bw = w; a.kpad = round_up(taps * c, kChunkK); a.n_total = c; a.bn = 0;
  a.bias = bias; a.flags = EPI_RES16 | EPI_OUT16; a.res16 = x; a.ldr16 = c; a.out16 = out; a.ld16 = c;
  // 19 taps on the position-windowed conv (each position's rows loaded once per
  // tile, the taps gathered on chip), else the gather-GEMM
  const int r = launch_conv_ts<__nv_bfloat16>(a, batch, n, n, st);
  if (r != 1) return r;
  return launch_gemm<__nv_bfloat16>(a, st);
}

int sb_offset_attention(const void* q, const void* k, const void* v, const float* table, int table_rows,
                        const int32_t* offset_map, int batch, int len, int heads, int head_dim, void* out,
                        void* stream) {
  if (!q || !k || !v || !table || !offset_map || !out || batch < 0 || len <= 0 || heads <= 0)
    return fail(SB_ERR_INVALID_ARG, "offset attention: bad args");
  if (batch == 0) return SB_OK;
  AttnArgs a{};
  a.q = q; a.k = k; a.v = v;
  a.pos_stride = (long long)len * heads * head_dim; a.row_stride = (long long)heads * head_dim; a.head_stride = head_dim;
  a.out = out; a.out_pos_stride = a.pos_stride; a.out_row_stride = a.row_stride; a.out_head_stride = head_dim;
  a.B = batch; a.S = len; a.H = heads; a.D = head_dim; a.ntok = 0;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  a.mode = BIAS_OFFSET; a.table = table; a.table_rows = table_rows; a.offset_map = offset_map;
  return launch_attention<__nv_bfloat16>(a, (cudaStream_t)stream);
}

}  // extern "C"
