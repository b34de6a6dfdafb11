/*
 * shrimp_b200 — C ABI of the B200-native Shrimp leaf-evaluation forward.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), enqueues its kernels on that stream without any host
 * synchronisation, and returns an sb_status. No exceptions cross the ABI and no
 * kernel traps: a device-side fault condition (out-of-range neighbour index, a
 * bounded wait that gave up) sets bits in the caller's status word instead.
 * The caller owns every buffer (inputs, outputs, weights, workspace); the
 * library never allocates or frees device memory.
 *
 * Conventions
 *   - "f16 rows": row-major IEEE half matrices; weights of the tensor-core
 *     layers are packed K-major as [N][Kpad] halves with Kpad a multiple of 64
 *     (see sb_pack_hex_conv_weight / sb_pack_linear_weight).
 *   - Sequence layout: every position owns S = 8 + Npad consecutive rows, the 8
 *     summary tokens first, then its Npad cells (reference model.py:905-926).
 *   - dtype codes: SB_F32, SB_F16, SB_BF16, SB_I64, SB_I32, SB_U8 (also bool),
 *     SB_I16, SB_U16.
 *
 * Reference interfaces replaced (paths inside Cmiller132/hexo-bot):
 *   packages/shrimp/python/shrimp/model.py            ShrimpNet and its blocks
 *   packages/shrimp/python/shrimp/_triton_conv.py     shrimp::hex_conv, shrimp::hex_conv_ln
 *   packages/shrimp/python/shrimp/_triton_attn.py     shrimp::attn_pair
 *   packages/shrimp/python/shrimp/losses.py           decode_binned_value / decode_moves_left
 *   packages/shrimp/python/shrimp/inference.py        ShrimpEvaluator._decode_group
 */
#ifndef SHRIMP_B200_H_
#define SHRIMP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_ABI_VERSION 1
#define SB_MAX_BLOCKS 32
#define SB_NUM_TOKENS 8
#define SB_NUM_FEATURES 15
#define SB_VALUE_BINS 65
#define SB_BIAS_ROWS 237      /* learned rows; row 237 is the pad-key row */
#define SB_LUT_W 35           /* clamped-offset LUT is SB_LUT_W x SB_LUT_W */

typedef enum {
  SB_OK = 0,
  SB_ERR_INVALID_ARG = 1,
  SB_ERR_UNSUPPORTED = 2,
  SB_ERR_CUDA = 3,
  SB_ERR_WORKSPACE = 4
} sb_status;

typedef enum {
  SB_F32 = 0,
  SB_F16 = 1,
  SB_BF16 = 2,
  SB_I64 = 3,
  SB_I32 = 4,
  SB_U8 = 5,
  SB_I16 = 6,
  SB_U16 = 7
} sb_dtype;

/* Status-word bits written by kernels (caller-provided int32 on the device). */
#define SB_DEV_ERR_TIMEOUT 1    /* a bounded mbarrier wait gave up */
#define SB_DEV_ERR_NBR_RANGE 2  /* a neighbour index was > Npad (treated as missing) */
#define SB_DEV_ERR_ROW_SIZE 4   /* a payload row has more nodes than its group's pad_to (truncated) */

/* ---- weights ----------------------------------------------------------------
 * Device pointers into caller-owned packed weights. "hw" = f16 [N][Kpad]
 * K-major; everything else fp32. */
typedef struct {
  const void* w1;  const float* b1;  const float* ln1_w; const float* ln1_b;
  const void* w2;  const float* b2;  const float* ln2_w; const float* ln2_b;
  const float* gamma;                 /* ls.gamma */
} sb_conv_block_weights;               /* ConvBlock, model.py:384-422 */

typedef struct {
  const float* ln1_w; const float* ln1_b;
  const void* wqkv;  const float* bqkv; /* [3C][C] = q_proj; k_proj; v_proj */
  const void* wo;    const float* bo;
  const float* gamma_attn;
  const float* ln2_w; const float* ln2_b;
  const void* w1;    const float* b1;   /* fc1 [2C][C] */
  const void* w2;    const float* b2;   /* fc2 [C][2C] */
  const float* gamma_mlp;
  const float* bias_table;              /* [238][H]: rows 0..236 = table rounded to f16, row 237 = -3e4 */
} sb_attn_block_weights;               /* AttnBlock, model.py:497-514 */

typedef struct {
  int channels;
  int heads;
  int num_blocks;
  char layout[SB_MAX_BLOCKS + 1];       /* 'C' / 'A', ends with 'A' */
  const void* stem_w;  const float* stem_b;   /* stem: Kpad over 7 taps x 16 (15 features + 0) */
  const float* stem_ln_w; const float* stem_ln_b;
  const float* tokens;                  /* [8][C] */
  const void* tokens_ln16;              /* [8][C] f16 = LN1 of the first attention block applied to tokens */
  const float* ln_final_w; const float* ln_final_b;
  const void* policy_conv_w; const float* policy_conv_b;
  const float* policy_head_w; const float* policy_head_b;  /* [C], [1] */
  const float* value_red_wT; const float* value_red_b;   /* [3C][C], [C] */
  const float* value_head_wT; const float* value_head_b; /* [C][65], [65] */
  const float* ml_red_wT; const float* ml_red_b;
  const float* ml_head_wT; const float* ml_head_b;
  const uint8_t* lut;                   /* [35*35] clamped-offset -> bias row */
  sb_conv_block_weights conv[SB_MAX_BLOCKS];
  sb_attn_block_weights attn[SB_MAX_BLOCKS];
} sb_net;

typedef struct {
  const void* feats;  int feats_dtype;  /* (B, Npad, 15) f32 / f16 / bf16 */
  const void* nbr;    int nbr_dtype;    /* (B, Npad, 6) i64 / i32 / u16; missing = Npad, -1 or 0xFFFF */
  const void* mask;   int mask_dtype;   /* (B, Npad) bool / u8 */
  const void* coords; int coords_dtype; /* (B, Npad, 2) i64 / i32 / i16 */
  int batch;
  int npad;
} sb_inputs;

typedef struct {
  float* policy;        /* (B, Npad) logits, pad rows 0 */
  float* value_logits;  /* (B, 65) */
  float* value;         /* (B) decoded scalar, or NULL */
  float* ml_logits;     /* (B, 65) moves-left logits, or NULL (not requested) */
  float* moves_left;    /* (B) decoded moves-left, or NULL */
  int32_t* status;      /* device status word (SB_DEV_ERR_* bits), or NULL */
} sb_outputs;

/* ---- library ------------------------------------------------------------- */
int sb_abi_version(void);
/* Copies the last host-side error message of the calling thread. */
int sb_last_error(char* buf, size_t len);

/* ---- whole forward: ShrimpNet.forward_policy_value (model.py:972-1003) ---- */
/* Bytes of workspace sb_forward_policy_value needs for (B, Npad). */
int sb_forward_workspace_bytes(const sb_net* net, int batch, int npad, size_t* bytes);
int sb_forward_policy_value(const sb_net* net, const sb_inputs* in, sb_outputs* out, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ---- serve payload: ShrimpEvaluator.submit_payload + result ---------------
 * (inference.py:509-604, 807-863, 865-1042; wire ABI shrimp-rs payload.rs:108-158)
 * The evaluator's request, already on the device: rows are positions, sorted
 * by node count (largest first), their support nodes concatenated (CSR). */
typedef struct {
  const void* node_feats; int feats_dtype;  /* (total_nodes, 15) f16 on the wire (f32 / bf16 accepted) */
  const int16_t* node_qr;                   /* (total_nodes, 2) hex coordinates (q, r) */
  const uint16_t* nbr;                      /* (total_nodes, 6) row-local neighbour index, 0xFFFF = missing */
  const int64_t* row_offsets;               /* (batch + 1) first node of each row; last = total_nodes */
  const int32_t* legal_counts;              /* (batch) legal-prefix length of each row */
  const int64_t* prior_offsets;             /* (batch) sum of legal_counts over the rows before */
  int batch;
} sb_payload;

/* The reply, on the device (the caller copies it to the wire bytes). */
typedef struct {
  float* values;         /* (batch) decoded value, clamped to [-1, 1] (values_bytes) */
  float* priors;         /* (sum legal_counts) softmax over each row's legal prefix, row order (priors_bytes) */
  float* moves_left;     /* (batch) decoded moves-left in [0, 209] (moves_left_bytes), or NULL */
  float* priors_logits;  /* (sum legal_counts) raw policy logits, same layout (priors_logits_bytes), or NULL */
  int32_t* status;       /* device status word (SB_DEV_ERR_* bits), or NULL */
} sb_reply;

/* One forward group: rows [start, end) padded to pad_to cells. */
typedef struct { int start, end, pad_to; } sb_group;

/* plan_groups (inference.py:201-223) on HOST row offsets: padding-aware
 * grouping of the size-sorted rows; pad_to = node count of the group's first
 * row rounded up to `quant` (>= quant); a group stops before the pair ceiling
 * (rows x (pad_to + 8)^2 > pair_ceiling) or before a row smaller than
 * pad_to - max(quant, int(waste_fraction * pad_to)). The reference uses
 * quant 64, waste_fraction 0.18, pair_ceiling 3.8e7. `groups` holds room for
 * `batch` entries. Rows out of size order are rejected. */
int sb_plan_groups(const int64_t* row_offsets, int batch, int quant, double waste_fraction, double pair_ceiling,
                   sb_group* groups, int* num_groups);
int sb_evaluate_workspace_bytes(const sb_net* net, const sb_group* groups, int num_groups, size_t* bytes);
/* Every group's forward straight from the CSR payload: the support rows are
 * unpacked and padded on the device (no host pack), attention skips each
 * position's dead key and query tiles, and the heads kernel writes the reply
 * (decoded value, moves-left, legal-prefix priors and logits). Groups are
 * independent and run on up to four lanes: `stream` and three auxiliary
 * streams of the calling host thread (created on its first call on a device
 * and kept for the life of the thread; not recreated after cudaDeviceReset),
 * forked from and joined back into `stream` by events, so the call is
 * ordered on `stream` as one unit and may be captured into a CUDA graph.
 * Each lane has its own slice of the workspace (sb_evaluate_workspace_bytes
 * sums them). */
int sb_evaluate_payload(const sb_net* net, const sb_payload* payload, const sb_group* groups, int num_groups,
                        sb_reply* reply, void* workspace, size_t workspace_bytes, void* stream);

/* ---- index tables (model.py:860-863 gather_idx; model.py:762-792 _build_pair_u8) */
/* gather_idx_out (B, Npad, 7) int32 row-local: tap 0 = self, taps 1..6 = nbr,
 * missing -> Npad (the reference's convention). */
int sb_build_gather_index(const void* nbr, int nbr_dtype, int batch, int npad, int32_t* gather_idx_out,
                          int32_t* status, void* stream);
/* pair_out (B, S, S) uint8, S = 8 + Npad: bias row of every (query, key). */
int sb_build_pair_u8(const void* coords, int coords_dtype, const void* mask, int mask_dtype, int batch,
                     int npad, const uint8_t* lut, uint8_t* pair_out, void* stream);

/* ---- kernel-op boundary (torch.library ops of the reference) ------------- */
/* shrimp::hex_conv (_triton_conv.py:93-128): out = (gather7(x) @ W + b) * mask.
 * x (B, Npad, Cin) f16, gather_idx (B, Npad, 7) int32 row-local (Npad = zero
 * row), mask (B, Npad) u8, w packed by sb_pack_hex_conv_weight, out f16. */
int sb_hex_conv(const void* x, const int32_t* gather_idx, const uint8_t* mask, const void* w_packed,
                const float* bias, int batch, int npad, int cin, int cout, void* out, void* workspace,
                size_t workspace_bytes, void* stream);
/* shrimp::hex_conv_ln (_triton_conv.py:198-239): LayerNorm(conv) (+ReLU) * mask. */
int sb_hex_conv_ln(const void* x, const int32_t* gather_idx, const uint8_t* mask, const void* w_packed,
                   const float* bias, const float* ln_w, const float* ln_b, float eps, int relu, int batch,
                   int npad, int cin, int cout, void* out, void* workspace, size_t workspace_bytes,
                   void* stream);
/* sb_hex_conv without a caller workspace (no counterpart in the reference).
 * For callers that cannot hand the library device memory at call time -
 * e.g. code that must not allocate between steps of a serving loop, or a
 * host that owns no allocator for scratch - the scratch lives in a fixed
 * 8 MiB device array inside the library: batch * npad must be <= 262,141
 * rows, larger calls fail with SB_ERR_UNSUPPORTED. The library allocates
 * nothing (no cudaMalloc / cudaFree). The first call on each device resolves
 * the array's address (set-up; make it before any stream capture) and keeps
 * it for the life of the process (it is not refreshed after cudaDeviceReset);
 * nothing in the scratch needs to start at zero (each call writes what it
 * reads). Calls share the one array per device, so calls that overlap in time
 * on the same device (different streams or threads) race: serialise them.
 * Same results as sb_hex_conv. */
int sb_hex_conv_noalloc(const void* x, const int32_t* gather_idx, const uint8_t* mask, const void* w_packed,
                        const float* bias, int batch, int npad, int cin, int cout, void* out, void* stream);
/* Workspace for sb_hex_conv / sb_hex_conv_ln, and the size of a plan. */
int sb_hex_conv_workspace_bytes(int batch, int npad, size_t* bytes);
/* Planned hex_conv for callers that run many convs over one neighbour table
 * (the reference's trunk calls shrimp::hex_conv / hex_conv_ln once per conv
 * layer with the same nbr, _triton_conv.py:93-128, 198-239; model.py:346-370).
 * sb_hex_conv_plan builds the per-table state once into `plan` (as many bytes
 * as sb_hex_conv_workspace_bytes gives): absolute gather rows, the row mask
 * and, for batches of >= 1024 positions of <= 81 cells, the hex-grid slots.
 * For such batches it synchronises `stream` once to read whether the cells
 * lie on the hex lattice (*lattice = 1; else 0) - make it outside stream
 * capture. Each planned conv
 * is then a single kernel launch (the grid conv when lattice = 1 and
 * cin == cout in {64, 128}, else the windowed conv / gather-GEMM); pass the
 * `lattice` value the plan returned. Results equal sb_hex_conv /
 * sb_hex_conv_ln on the same table. The plan stays valid while gather_idx and
 * mask are unchanged; the planned calls only read it. */
int sb_hex_conv_plan(const int32_t* gather_idx, const uint8_t* mask, int batch, int npad, void* plan,
                     size_t plan_bytes, int* lattice, void* stream);
int sb_hex_conv_planned(const void* x, const void* plan, size_t plan_bytes, int lattice, const void* w_packed,
                        const float* bias, int batch, int npad, int cin, int cout, void* out, void* stream);
int sb_hex_conv_ln_planned(const void* x, const void* plan, size_t plan_bytes, int lattice, const void* w_packed,
                           const float* bias, const float* ln_w, const float* ln_b, float eps, int relu, int batch,
                           int npad, int cin, int cout, void* out, void* stream);
/* shrimp::attn_pair (_triton_attn.py:132-171): q, k, v (B, H, S, D) f16 with
 * unit stride on D, pair (B, S, S) uint8, table2 (238, H) f32 (the op rounds it
 * to f16: pass f16-representable values for identical results), seq_lens (B)
 * int32 live lengths or NULL (= S): keys >= seq_lens[b] are skipped and query
 * rows >= seq_lens[b] are written as zeros (padding; the caller masks them),
 * out (B, H, S, D). */
int sb_attn_pair(const void* q, const void* k, const void* v, const uint8_t* pair, const float* table2,
                 const int32_t* seq_lens, int batch, int heads, int seq, int head_dim, void* out, void* stream);

/* ---- weight packing ------------------------------------------------------ */
/* HexNodeConv weight (taps, Cin, Cout) fp32 -> f16 [Cout][Kpad], Kpad =
 * roundup(taps * cin_pad, 64), channel c >= Cin of each tap zero. */
int sb_pack_hex_conv_weight(const float* w, int taps, int cin, int cin_pad, int cout, void* out, void* stream);
/* nn.Linear weight (N, K) fp32 -> f16 [N][Kpad]. */
int sb_pack_linear_weight(const float* w, int n, int k, void* out, void* stream);

/* ---- decode (losses.py:40-61, inference.py:998-1042) ---------------------- */
int sb_decode_binned(const float* logits, int batch, float scale, float offset, float* out, void* stream);
/* priors_out[row_offsets[b] + i] = softmax(policy[b, :legal[b]])[i]. */
int sb_legal_prefix_softmax(const float* policy, int batch, int npad, const int32_t* legal_counts,
                            const int64_t* row_offsets, float* priors_out, void* stream);

/* ---- microbench kernels (BASELINE configs 2 and 3) ------------------------ */
/* out = relu(gather_T(x) @ W + b + x); x (B, N, C) bf16, nbr (N, T) int32 (-1 = off support),
 * W packed [C][Kpad] bf16. Workspace: B * N * T int32 plus 64 bytes. */
int sb_raytap_conv(const void* x, const int32_t* nbr, int taps, const void* w_packed, const float* bias,
                   int batch, int n, int c, void* out, void* workspace, size_t workspace_bytes, void* stream);
/* out = softmax(Q.K^T / sqrt(d) + table[offset_map, h]) V; q, k, v, out (B, L, H*d) bf16. */
int sb_offset_attention(const void* q, const void* k, const void* v, const float* table, int table_rows,
                        const int32_t* offset_map, int batch, int len, int heads, int head_dim, void* out,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SHRIMP_B200_H_ */
