// Fused multi-head attention backward for sm_100a (gko::fused_sdpa_bwd and the
// packed variable-length variant).
//
// Given q, k, v, the forward output O, its lse and dO, computes dq, dk, dv of
//   O = softmax(mask(softcap(scale * q k^T + bias))) v
// with the reference's recompute formulation (eval/kernels/fused_sdpa.py:159-496,
// 668-770): delta = rowsum(O * dO); P = exp(logits - lse); dP = dO v^T;
// dS = P * (dP - delta) [* softcap derivative]; dv = P^T dO; dk = scale dS^T q;
// dq = scale dS k. Three launches on the caller's stream:
//
//   1. prep      one CTA per 64-query block: -delta and -lse*log2(e) into the
//                workspace (padded rows get 0 / -inf, so they contribute nothing),
//                and zeroes the block's fp32 dq accumulator.
//   2. main      one CTA per 128-key tile of one kv head; it steps over every (query
//                head of the GQA group, 64-query block) the masks allow.
//   3. convert   dq = scale * accumulator, cast to the input dtype.
//
// The main kernel is laid out around two costs of B200: shared-memory bandwidth
// (about 128 B per clock per SM, which limits MMAs that read both operands from shared
// memory at N <= 64) and the latency of a hand-off between warps through an mbarrier
// (a few hundred cycles, more after a tcgen05.commit). K is copied once into TMEM and is
// the A operand (TS form) of S^T = K Q^T; dV and dK take P^T / dS^T from TMEM; dQ^T has
// its own TMEM buffer, so the MMA for the next step's dP^T never waits for dQ^T to be
// drained, and the dS^T smem tile is double buffered. dQ^T leaves TMEM through registers
// as fp32 reductions into L2 (no shared-memory staging).
// TMEM columns: K [0, 64)  dQ^T [64, 128)  dV [128, 256)  dK [256, 384)
//               S^T|P^T [384, 448)  dP^T|dS^T [448, 512)
//   warp 13    MMA issuer. Step j, in issue order:
//                dV += P^T_j dO_j        (A = P^T in TMEM, B = dO_j MN-major)
//                S^T_{j+1} = K Q_{j+1}^T (A = K in TMEM) — the S columns are free once dV_j is issued
//                dK += dS^T_j Q_j        (A = dS^T in TMEM)
//                dP^T_{j+1} = V dO_{j+1}^T (both from smem) — the dP columns are free once dK_j is issued
//                dQ^T_j = K^T dS^T_j     (both from smem, MN-major) once warps 8-11 have read dQ^T_{j-1}
//   warp 12    TMA producer: K, V once; Q_j, dO_j, -lse_j, -delta_j per step (3 stages).
//   warps 0-7  compute: warp w owns key rows 32 (w & 3) .. +31 (its TMEM lane quarter) and
//              query columns 32 (w >> 2) .. +31: first K (w < 4) into TMEM; then per step
//              P^T = 2^(s * scale * log2 e - lse * log2 e) over S^T (bf16/f16 pairs) and
//              dS^T = P^T (dP^T - delta) over dP^T and into smem dS tile j & 1.
//              At the end dk = scale * dK (half the columns each).
//   warps 8-11 one head-dim row of dQ^T_j per thread: 64 fp32 reductions (red.global.add)
//              into the row-major [queries][D] accumulator; at the end dv = dV.
// Registers: 16 warps x 128 at launch; the compute warpgroups rise to 152, the drain
// warpgroup drops to 112 and the producer/MMA warpgroup to 96
// (128 x (2 x 152 + 112 + 96) = 65536 = 512 x 128).
#include <mutex>
#include <type_traits>

#include "host_common.h"
#include "sm100_ptx.cuh"

namespace gko {
namespace fmha_bwd {

constexpr int kBN = 128;  // keys per CTA (one per TMEM lane)
constexpr int kBM = 64;   // queries per step
constexpr int kThreads = 512;
constexpr int kDrainWarp0 = 8;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kStages = 3;
constexpr uint32_t kRegsCompute = 152;
constexpr uint32_t kRegsDrain = 112;
constexpr uint32_t kRegsControl = 96;
static_assert(128 * (2 * kRegsCompute + kRegsDrain + kRegsControl) <= 512 * 128, "register split exceeds the launch");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmK = 0, kTmDQ = 64, kTmDV = 128, kTmDK = 256, kTmS = 384, kTmDP = 448;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  int hq, hkv, group;
  int sq, sk;     // dense per-batch lengths
  int zh_kv;      // batch (or sequences) x kv heads
  float scale, scale_log2, softcap;
  int causal, window;
  const void* bias;
  int bias_mode, bias_dtype, bias_z;
  int64_t b_sz, b_sh, b_sq, b_sk;
  // workspace, indexed by 64-query block ("tile": per head, consecutive blocks of rows)
  float* dq_acc;      // [tiles][64 queries][D], row-major fp32
  const float* nl;    // [tiles][64]  -lse * log2(e), -inf for padded / empty rows
  const float* nd;    // [tiles][64]  -rowsum(O * dO)
  int64_t tiles_per_head;
  void* dk;
  int64_t dk_sz, dk_sh, dk_ss;
  void* dv;
  int64_t dv_sz, dv_sh, dv_ss;
  const int* cu_q;
  const int* cu_k;
  int total_q, total_k;  // varlen: packed query / key tokens (every row index stays below them)
  unsigned* status;
};

// Parameters of the prep and convert kernels (one CTA per 64-query block of one query head).
struct RowParams {
  int hq, sq, zh;
  const void* o;
  int64_t o_sz, o_sh, o_ss;
  const void* dout;
  int64_t do_sz, do_sh, do_ss;
  const float* lse;
  int64_t lse_stride_h;  // dense: sq; varlen: total query tokens
  float* dq_acc;
  float* nl;
  float* nd;
  int64_t tiles_per_head;
  void* dq;
  int64_t dq_sz, dq_sh, dq_ss;
  float scale;
  const int* cu_q;
  int total_q;  // varlen: packed query tokens
};

// Rows [row0, row0 + len) of sequence b (varlen), clamped to the packed tokens [0, total):
// whatever cu_seqlens hold, no row index formed from them leaves the tensors.
__device__ __forceinline__ void varlen_rows(const int* cu, int b, int total, int& row0, int& len) {
  const int a = min(max(cu[b], 0), total);
  const int e = min(max(cu[b + 1], a), total);
  row0 = a;
  len = e - a;
}

// First 64-query block of sequence b in a head's run of blocks (varlen), from its clamped first
// row a: blocks of consecutive sequences never overlap because ceil(a/64) + ceil(l/64) <=
// ceil((a+l)/64) + 1, and with a + l <= total every block index stays below
// ceil(total/64) + batch, inside the workspace's ceil(total/64) + batch + 1 blocks per head.
__device__ __forceinline__ int64_t varlen_block_base(int row_q0, int b) {
  return (int64_t)((row_q0 + kBM - 1) / kBM) + b;
}

__device__ __forceinline__ float bias_at(const Params& p, int z, int h, int q, int k) {
  const int64_t off = (int64_t)(z % p.bias_z) * p.b_sz + (int64_t)h * p.b_sh + (int64_t)q * p.b_sq +
                      (int64_t)k * p.b_sk;
  if (p.bias_dtype == GKO_F32) return __ldg(reinterpret_cast<const float*>(p.bias) + off);
  if (p.bias_dtype == GKO_BF16)
    return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(p.bias) + off));
  return __half2float(__ldg(reinterpret_cast<const __half*>(p.bias) + off));
}

template <int D>
struct Layout {
  static constexpr uint32_t kChunkKV = 128 * 128;  // [128 rows][128 B]
  static constexpr uint32_t kChunkQ = 64 * 128;    // [64 rows][128 B]
  static constexpr uint32_t kTileKV = (D / 64) * kChunkKV;
  static constexpr uint32_t kTileQ = (D / 64) * kChunkQ;
  static constexpr uint32_t kK = 0;
  static constexpr uint32_t kV = kTileKV;
  static constexpr uint32_t kStage0 = 2 * kTileKV;  // stage s: Q at +0, dO at +kTileQ
  static constexpr uint32_t kStageBytes = 2 * kTileQ;
  static constexpr uint32_t kDS = kStage0 + kStages * kStageBytes;  // 2 x [128 keys][64 q] bf16, SW128
  static constexpr uint32_t kDSBytes = kBN * 128;
  static constexpr uint32_t kRow = kDS + 2 * kDSBytes;  // per stage: -lse log2 e [64], -delta [64]
  static constexpr uint32_t kMeta = kRow + kStages * 512;
  static constexpr uint32_t kBytes = (1024 + kMeta + 256) > 122880 ? (1024 + kMeta + 256) : 122880;
  static_assert(kDS % 1024 == 0 && kStageBytes % 1024 == 0, "swizzled tiles need 1024-byte alignment");
  static_assert(1024 + kMeta + 256 <= 232448, "shared memory budget");
};

template <typename T, int D, bool VARLEN, bool EXTRA>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const Params p) {
  using L = Layout<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = make_idesc_f16(kBF16, kBN, kBM, false, false);  // S^T, dP^T
  constexpr uint32_t kIdescKV = make_idesc_f16(kBF16, kBN, D, false, true);    // dV, dK
  constexpr uint32_t kIdescQ = make_idesc_f16(kBF16, 128, kBM, true, true);    // dQ^T

  // ---------------------------------------------------------- block geometry
  const int bh = (int)blockIdx.y + (int)blockIdx.z * (int)gridDim.y;
  if (bh >= p.zh_kv) return;
  const int hk = bh % p.hkv;
  const int zb = bh / p.hkv;
  const int n0 = (int)blockIdx.x * kBN;  // first key of this CTA (sequence-local)
  int len_q, len_k, row_q0, row_k0;
  if constexpr (VARLEN) {
    varlen_rows(p.cu_q, zb, p.total_q, row_q0, len_q);
    varlen_rows(p.cu_k, zb, p.total_k, row_k0, len_k);
  } else {
    row_q0 = 0;
    len_q = p.sq;
    row_k0 = 0;
    len_k = p.sk;
  }
  if (n0 >= len_k) return;  // uniform across the CTA
  const int zc = VARLEN ? 0 : zb;
  // query range the masks allow for keys [n0, n0 + 128)
  int q_lo = 0, q_hi = len_q;
  if (p.causal) q_lo = max(q_lo, n0);
  if (p.window > 0) {
    q_lo = max(q_lo, n0 - p.window);
    q_hi = min(q_hi, n0 + kBN - 1 + p.window + 1);
  }
  const int jb_lo = q_lo / kBM;
  const int nq = q_hi > q_lo ? (q_hi + kBM - 1) / kBM - jb_lo : 0;
  const int n_steps = nq * p.group;
  const int64_t tile_base = VARLEN ? varlen_block_base(row_q0, zb) : 0;
  auto tile_of = [&](int hh, int jb) -> int64_t {  // workspace block of (query head, 64-query block)
    const int h = hk * p.group + hh;
    return (VARLEN ? (int64_t)h : (int64_t)zb * p.hq + h) * p.tiles_per_head + tile_base + jb;
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  T* dk_base;
  T* dv_base;
  if constexpr (VARLEN) {
    dk_base = reinterpret_cast<T*>(p.dk) + (int64_t)row_k0 * p.dk_ss + (int64_t)hk * p.dk_sh;
    dv_base = reinterpret_cast<T*>(p.dv) + (int64_t)row_k0 * p.dv_ss + (int64_t)hk * p.dv_sh;
  } else {
    dk_base = reinterpret_cast<T*>(p.dk) + (int64_t)zb * p.dk_sz + (int64_t)hk * p.dk_sh;
    dv_base = reinterpret_cast<T*>(p.dv) + (int64_t)zb * p.dv_sz + (int64_t)hk * p.dv_sh;
  }
  if (n_steps == 0) {  // no query sees these keys: dk = dv = 0
    for (int i = threadIdx.x; i < kBN * (D / 8); i += kThreads) {
      const int r = i / (D / 8), c = i % (D / 8);
      if (n0 + r < len_k) {
        reinterpret_cast<uint4*>(dk_base + (int64_t)(n0 + r) * p.dk_ss)[c] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(dv_base + (int64_t)(n0 + r) * p.dv_ss)[c] = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  // ---------------------------------------------------------- shared memory
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  const uint32_t sb = raw_addr + pad;
  uint8_t* sgen = smem_raw + pad;  // generic pointer to the same base
  const uint32_t smeta = sb + L::kMeta;
  const uint32_t bar_kv = smeta;            // K, V landed in smem (TMA)
  const uint32_t bar_kvtm = smeta + 8;      // K copied into TMEM (4 arrivals)
  const uint32_t bar_full = smeta + 16;     // [3]
  const uint32_t bar_empty = smeta + 40;    // [3]
  const uint32_t bar_sfull = smeta + 64;
  const uint32_t bar_pfull = smeta + 72;    // 8 arrivals
  const uint32_t bar_dpfull = smeta + 80;
  const uint32_t bar_dsfull = smeta + 88;   // 8 arrivals
  const uint32_t bar_dqfull = smeta + 96;
  const uint32_t bar_dqempty = smeta + 104;  // 4 arrivals
  const uint32_t bar_dsfree = smeta + 112;   // [2] per smem dS tile: dQ^T has read it
  const uint32_t bar_final = smeta + 128;
  const uint32_t bar_drain = smeta + 136;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + L::kMeta + 144);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + L::kMeta + 148);

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    mbar_init(bar_kvtm, 4);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar_full + 8 * i, 1);
      mbar_init(bar_empty + 8 * i, 1);
    }
    mbar_init(bar_sfull, 1);
    mbar_init(bar_pfull, 8);
    mbar_init(bar_dpfull, 1);
    mbar_init(bar_dsfull, 8);
    mbar_init(bar_dqfull, 1);
    mbar_init(bar_dqempty, 4);
    mbar_init(bar_dsfree, 1);
    mbar_init(bar_dsfree + 8, 1);
    mbar_init(bar_final, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_do);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= kProducerWarp) {
    setmaxnreg_dec<kRegsControl>();
    if (warp == kProducerWarp) {
      // ---------------------------------------------------------- TMA producer
      if (lane == 0) {
        mbar_arrive_expect_tx(bar_kv, 2 * L::kTileKV);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(sb + L::kK + c * L::kChunkKV, &tm_k, bar_kv, c * 64, row_k0 + n0, hk, zc);
          tma_load_4d(sb + L::kV + c * L::kChunkKV, &tm_v, bar_kv, c * 64, row_k0 + n0, hk, zc);
        }
        for (int j = 0; j < n_steps; ++j) {
          const int st = j % kStages;
          const uint32_t ph = (j / kStages) & 1;
          const int hh = j / nq;
          const int jb = jb_lo + j % nq;
          if (!wait_bounded(bar_empty + 8 * st, ph ^ 1, abort_flag, p.status, kStatusTimeoutProducer)) break;
          const uint32_t stage = sb + L::kStage0 + st * L::kStageBytes;
          const uint32_t full = bar_full + 8 * st;
          mbar_arrive_expect_tx(full, 2 * L::kTileQ + 512);
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            tma_load_4d(stage + c * L::kChunkQ, &tm_q, full, c * 64, row_q0 + jb * kBM, hk * p.group + hh, zc);
            tma_load_4d(stage + L::kTileQ + c * L::kChunkQ, &tm_do, full, c * 64, row_q0 + jb * kBM,
                        hk * p.group + hh, zc);
          }
          const int64_t t = tile_of(hh, jb);
          bulk_load(sb + L::kRow + st * 512, p.nl + t * kBM, kBM * 4, full);
          bulk_load(sb + L::kRow + st * 512 + 256, p.nd + t * kBM, kBM * 4, full);
        }
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------- MMA issuer
      if (lane == 0) {
        // Shared-memory descriptors are built once: a K step or a stage only adds a constant to
        // the 14-bit start-address field (every address here is below 256 KB, so it never
        // carries). Per-MMA descriptor arithmetic would otherwise cost the single issuing thread
        // more time than an N <= 128 MMA takes to execute.
        const uint64_t d_qk = make_sdesc_sw128(sb + L::kStage0, 16, 1024);           // Q / dO as K-major B
        const uint64_t d_qmn = make_sdesc_sw128(sb + L::kStage0, L::kChunkQ, 1024);  // Q / dO as MN-major B
        const uint64_t d_v = make_sdesc_sw128(sb + L::kV, 16, 1024);                 // V as K-major A
        const uint64_t d_kmn = make_sdesc_sw128(sb + L::kK, L::kChunkKV, 1024);      // K as MN-major A
        const uint64_t d_ds = make_sdesc_sw128(sb + L::kDS, 8192, 1024);             // dS^T tiles as MN-major B
        const uint32_t t_s = tmem_base + kTmS, t_dp = tmem_base + kTmDP, t_dv = tmem_base + kTmDV;
        const uint32_t t_dk = tmem_base + kTmDK, t_k = tmem_base + kTmK, t_dq = tmem_base + kTmDQ;
        constexpr uint32_t kStageU = L::kStageBytes >> 4, kTileQU = L::kTileQ >> 4, kDSU = L::kDSBytes >> 4;
        // K-major K step kk: +32 bytes inside a 64-element chunk, chunks kChunkQ / kChunkKV apart
        auto kmaj_q = [](int kk) -> uint32_t { return (uint32_t)(((kk >> 2) * L::kChunkQ + (kk & 3) * 32) >> 4); };
        auto kmaj_kv = [](int kk) -> uint32_t { return (uint32_t)(((kk >> 2) * L::kChunkKV + (kk & 3) * 32) >> 4); };
        // S^T_j = K Q_j^T: A = K (TMEM, packed pairs along d), B = Q_j (K-major)
        auto issue_s = [&](int j) {
          const uint64_t b = d_qk + (uint64_t)((j % kStages) * kStageU);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) mma_f16_ts(t_s, t_k + kk * 8, b + kmaj_q(kk), kIdescS, kk > 0 ? 1u : 0u);
          mma_commit(bar_sfull);
        };
        // dP^T_j = V dO_j^T: A = V (K-major smem), B = dO_j (K-major)
        auto issue_dp = [&](int j) {
          const uint64_t b = d_qk + (uint64_t)((j % kStages) * kStageU + kTileQU);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) mma_f16_ss(t_dp, d_v + kmaj_kv(kk), b + kmaj_q(kk), kIdescS, kk > 0 ? 1u : 0u);
          mma_commit(bar_dpfull);
        };
        bool ok = wait_bounded(bar_kvtm, 0, abort_flag, p.status, kStatusTimeoutMma);
        if (ok) ok = wait_bounded(bar_kv, 0, abort_flag, p.status, kStatusTimeoutMma);
        if (ok) ok = wait_bounded(bar_full, 0, abort_flag, p.status, kStatusTimeoutMma);
        if (ok) {
          tc_fence_after();
          issue_s(0);
          issue_dp(0);
        }
        for (int j = 0; j < n_steps && ok; ++j) {
          const uint64_t st_mn = d_qmn + (uint64_t)((j % kStages) * kStageU);  // Q_j (MN-major); dO_j at + kTileQU
          const uint32_t ph = j & 1;
          const uint32_t acc0 = j > 0 ? 1u : 0u;
          // P^T and dS^T are packed: the 16 columns of query group g sit at + 32 g
          // dV += P^T_j dO_j: B = dO_j as [q][d] (MN-major), 16 rows (2048 bytes) per K step
          ok = wait_bounded(bar_pfull, ph, abort_flag, p.status, kStatusTimeoutMma);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            mma_f16_ts(t_dv, t_s + (kk >> 1) * 32 + (kk & 1) * 8, st_mn + kTileQU + kk * 128, kIdescKV,
                       kk > 0 ? 1u : acc0);
          const bool next = j + 1 < n_steps;
          if (next) {
            ok = wait_bounded(bar_full + 8 * ((j + 1) % kStages), ((j + 1) / kStages) & 1, abort_flag, p.status,
                              kStatusTimeoutMma);
            if (!ok) break;
            tc_fence_after();
            issue_s(j + 1);  // after dV_j in issue order, so P^T_j has been read
          }
          // dK += dS^T_j Q_j
          ok = wait_bounded(bar_dsfull, ph, abort_flag, p.status, kStatusTimeoutMma);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            mma_f16_ts(t_dk, t_dp + (kk >> 1) * 32 + (kk & 1) * 8, st_mn + kk * 128, kIdescKV, kk > 0 ? 1u : acc0);
          mma_commit(bar_empty + 8 * (j % kStages));  // Q_j, dO_j, -lse_j, -delta_j no longer needed
          if (next) issue_dp(j + 1);                  // after dK_j in issue order, so dS^T_j has been read
          // dQ^T_j = K^T dS^T_j: A = K as [key][d] (MN-major over d; for D = 64 the second 64-row
          // chunk reads V and lands in TMEM lanes nobody reads), B = dS^T tile j & 1 [key][q]
          if (j > 0) {
            ok = wait_bounded(bar_dqempty, ph ^ 1, abort_flag, p.status, kStatusTimeoutMma);
            if (!ok) break;
            tc_fence_after();
          }
          const uint64_t b_ds = d_ds + (uint64_t)((j & 1) * kDSU);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk)
            mma_f16_ss(t_dq, d_kmn + kk * 128, b_ds + kk * 128, kIdescQ, kk > 0 ? 1u : 0u);
          mma_commit(bar_dqfull);
          mma_commit(bar_dsfree + 8 * (j & 1));
        }
        if (ok) mma_commit(bar_final);
        if (*abort_flag) {
          mma_commit(bar_drain);
          wait_for(bar_drain, 0, p.status, kStatusTimeoutDrain);
        }
      }
    }
  } else if (warp < kDrainWarp0) {
    setmaxnreg_inc<kRegsCompute>();
    // ------------------------------------------------------------ compute (key row x 32 query columns)
    const int quarter = warp & 3;
    const int cg = warp >> 2;  // query columns 32 cg .. 32 cg + 31; warps of cg 0 copy K into TMEM
    const int r = quarter * 32 + lane;
    const int kj = n0 + r;
    const bool row_valid = kj < len_k;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tm_row = tmem_base + lane_off;
    const uint64_t k2 = f2pack(p.scale_log2, p.scale_log2);
    bool ok = cg ? true : wait_bounded(bar_kv, 0, abort_flag, p.status, kStatusTimeoutSoftmax);
    if (ok && cg == 0) {
      // row r of K from the swizzled smem tile into TMEM as bf16/f16 pairs along d
      const uint8_t* src = sgen + L::kK + r * 128;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 x = *reinterpret_cast<const uint4*>(src + c * L::kChunkKV + ((i ^ (r & 7)) << 4));
          w[4 * i] = x.x;
          w[4 * i + 1] = x.y;
          w[4 * i + 2] = x.z;
          w[4 * i + 3] = x.w;
        }
        tmem_st32(tm_row + kTmK + c * 32, w);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_kvtm);
    }
    for (int j = 0; j < n_steps && ok; ++j) {
      const uint32_t ph = j & 1;
      const int jb = jb_lo + j % nq;
      const int hh = j / nq;
      const int q0 = jb * kBM + cg * 32;  // first query of this warp's columns
      const float2* nl2 = reinterpret_cast<const float2*>(sgen + L::kRow + (j % kStages) * 512) + cg * 16;
      const float2* nd2 = reinterpret_cast<const float2*>(sgen + L::kRow + (j % kStages) * 512 + 256) + cg * 16;
      // the stage's -lse / -delta rows were written by the bulk copy: observe its barrier
      // here too (it completed before S^T_j; the stage is refilled only after dS_j)
      if (!wait_bounded(bar_sfull, ph, abort_flag, p.status, kStatusTimeoutSoftmax) ||
          !wait_bounded(bar_full + 8 * (j % kStages), (j / kStages) & 1, abort_flag, p.status,
                        kStatusTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float pv[32];  // S^T row, then P^T row
      {
        uint32_t su[32];
        tmem_ld32p(tm_row + kTmS + cg * 32, su);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) pv[c] = __uint_as_float(su[c]);
      }
      float gsc[EXTRA ? 32 : 1];  // softcap derivative
      if constexpr (EXTRA) {
        const int h = hk * p.group + hh;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int qi = q0 + c;
          float x = pv[c] * p.scale;
          if (p.bias_mode != GKO_BIAS_NONE && row_valid && qi < len_q) x += bias_at(p, zb, h, qi, kj);
          float g = 1.f;
          if (p.softcap > 0.f) {
            const float u = x / p.softcap;
            const float t = tanhf(fminf(fmaxf(u, -15.f), 15.f));
            g = (u > -15.f && u < 15.f) ? 1.f - t * t : 0.f;
            x = p.softcap * t;
          }
          bool keep = row_valid;
          if (p.causal) keep = keep && (kj <= qi);
          if (p.window > 0) keep = keep && (kj - qi <= p.window) && (qi - kj <= p.window);
          const float2 nlp = nl2[c >> 1];
          pv[c] = keep ? fast_exp2(fmaf(x, kLog2e, (c & 1) ? nlp.y : nlp.x)) : 0.f;
          gsc[c] = g;
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float2 nlp = nl2[c >> 1];
          float a, bb;
          f2unpack(fma2(f2pack(pv[c], pv[c + 1]), k2, f2pack(nlp.x, nlp.y)), a, bb);
          pv[c] = fast_exp2(a);
          pv[c + 1] = fast_exp2(bb);
        }
        // keys past the end, and (causal) queries before the key, get P = 0
        const int lim = row_valid ? (p.causal ? kj - q0 : 0) : 32;
        if (lim > 0) {
#pragma unroll
          for (int c = 0; c < 32; ++c) pv[c] = (c < lim) ? 0.f : pv[c];
        }
      }
      {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[c] = Cvt<T>::pack(pv[2 * c], pv[2 * c + 1]);
        tmem_st16(tm_row + kTmS + cg * 32, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_pfull);
      }
      // dS^T = P^T (dP^T - delta)
      if (!wait_bounded(bar_dpfull, ph, abort_flag, p.status, kStatusTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t dsu[32];
      tmem_ld32p(tm_row + kTmDP + cg * 32, dsu);
      tmem_wait_ld();
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const float2 ndp = nd2[c >> 1];
        const uint64_t t = add2(f2pack(__uint_as_float(dsu[c]), __uint_as_float(dsu[c + 1])), f2pack(ndp.x, ndp.y));
        float a, bb;
        f2unpack(mul2(f2pack(pv[c], pv[c + 1]), t), a, bb);
        if constexpr (EXTRA) {
          a *= gsc[c];
          bb *= gsc[c + 1];
        }
        pk[c >> 1] = Cvt<T>::pack(a, bb);
      }
      tmem_st16(tm_row + kTmDP + cg * 32, pk);
      // dS^T row r into smem tile j & 1 ([128 keys][64 q], 16-byte chunk i at (i ^ (r & 7))),
      // once dQ^T_{j-2} has finished reading that tile
      if (j >= 2 &&
          !wait_bounded(bar_dsfree + 8 * (j & 1), ((j - 2) >> 1) & 1, abort_flag, p.status, kStatusTimeoutSoftmax)) {
        ok = false;
        break;
      }
      const uint32_t ds_row = sb + L::kDS + (j & 1) * L::kDSBytes + r * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ci = cg * 4 + i;
        st_shared_v4(ds_row + ((ci ^ (r & 7)) << 4), pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      fence_proxy_async_smem();
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_dsfull);
    }
    // ------------------------------------------------------------ dk = scale * dK (columns cg * D/2 ..)
    if (ok) ok = wait_bounded(bar_final, 0, abort_flag, p.status, kStatusTimeoutSoftmax);
    if (ok) {
      tc_fence_after();
      T* row = dk_base + (int64_t)kj * p.dk_ss;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        const int col = cg * (D / 2) + c * 32;
        uint32_t v[32];
        tmem_ld32(tm_row + kTmDK + col, v);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          w[e] = Cvt<T>::pack(__uint_as_float(v[2 * e]) * p.scale, __uint_as_float(v[2 * e + 1]) * p.scale);
        if (row_valid) {
          uint4* dst = reinterpret_cast<uint4*>(row + col);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
    }
    tc_fence_before();
  } else {
    setmaxnreg_dec<kRegsDrain>();
    // ------------------------------------------------------------ dQ^T drain (one head-dim row per thread)
    const int wq = warp - kDrainWarp0;
    const int dr = wq * 32 + lane;  // TMEM lane: dQ^T row d, later dV row (key)
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tm_row = tmem_base + lane_off;
    bool ok = true;
    for (int j = 0; j < n_steps; ++j) {
      if (!wait_bounded(bar_dqfull, j & 1, abort_flag, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t v[kBM];
      tmem_ld32p(tm_row + kTmDQ, v);
      tmem_ld32p(tm_row + kTmDQ + 32, v + 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_dqempty);
      if (dr < D) {
        // accumulator block: row-major [64 queries][D]; a warp's 32 rows d are 128 contiguous bytes
        float* dst = p.dq_acc + tile_of(j / nq, jb_lo + j % nq) * (kBM * D) + dr;
#pragma unroll
        for (int q = 0; q < kBM; ++q) atomicAdd(dst + q * D, __uint_as_float(v[q]));
      }
    }
    // ------------------------------------------------------------ dv = dV
    if (ok) ok = wait_bounded(bar_final, 0, abort_flag, p.status, kStatusTimeoutEpilogue);
    if (ok) {
      tc_fence_after();
      const int kj = n0 + dr;
      T* row = dv_base + (int64_t)kj * p.dv_ss;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t w32[32];
        tmem_ld32(tm_row + kTmDV + c * 32, w32);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) w[e] = Cvt<T>::pack(__uint_as_float(w32[2 * e]), __uint_as_float(w32[2 * e + 1]));
        if (kj < len_k) {
          uint4* o = reinterpret_cast<uint4*>(row + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) o[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
    }
    tc_fence_before();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ prep: -delta, -lse log2 e, zero dq
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Cvt<T>::to_f32(e[i]);
}

template <typename T, int D, bool VARLEN>
__global__ void __launch_bounds__(256) fmha_bwd_prep_kernel(const RowParams p) {
  const int bh = (int)blockIdx.y + (int)blockIdx.z * (int)gridDim.y;
  if (bh >= p.zh) return;
  const int h = bh % p.hq;
  const int zb = bh / p.hq;
  const int jb = blockIdx.x;
  int row_q0 = 0, len_q = p.sq;
  int64_t base = 0;
  if constexpr (VARLEN) {
    varlen_rows(p.cu_q, zb, p.total_q, row_q0, len_q);
    base = varlen_block_base(row_q0, zb);
  }
  if (jb * kBM >= len_q) return;
  const int64_t tile = (VARLEN ? (int64_t)h : (int64_t)bh) * p.tiles_per_head + base + jb;
  // zero this block's dq accumulator
  uint4* acc = reinterpret_cast<uint4*>(p.dq_acc + tile * (kBM * D));
  for (int i = threadIdx.x; i < kBM * D / 4; i += 256) acc[i] = make_uint4(0, 0, 0, 0);
  // 4 threads per query row, D / 4 elements each
  const int row = threadIdx.x >> 2, part = threadIdx.x & 3;
  const int qi = jb * kBM + row;
  float s = 0.f;
  if (qi < len_q) {
    const T* o;
    const T* g;
    if constexpr (VARLEN) {
      o = reinterpret_cast<const T*>(p.o) + (int64_t)(row_q0 + qi) * p.o_ss + (int64_t)h * p.o_sh;
      g = reinterpret_cast<const T*>(p.dout) + (int64_t)(row_q0 + qi) * p.do_ss + (int64_t)h * p.do_sh;
    } else {
      o = reinterpret_cast<const T*>(p.o) + (int64_t)zb * p.o_sz + (int64_t)h * p.o_sh + (int64_t)qi * p.o_ss;
      g = reinterpret_cast<const T*>(p.dout) + (int64_t)zb * p.do_sz + (int64_t)h * p.do_sh +
          (int64_t)qi * p.do_ss;
    }
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float a[8], b[8];
      load8(o + part * (D / 4) + c * 8, a);
      load8(g + part * (D / 4) + c * 8, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(a[e], b[e], s);
    }
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if (part == 0) {
    float nl = -INFINITY;
    if (qi < len_q) {
      const float l = VARLEN ? p.lse[(int64_t)h * p.lse_stride_h + row_q0 + qi]
                             : p.lse[(int64_t)bh * p.lse_stride_h + qi];
      nl = (l == -INFINITY) ? -INFINITY : -l * kLog2e;
    }
    p.nl[tile * kBM + row] = nl;
    p.nd[tile * kBM + row] = (qi < len_q) ? -s : 0.f;
  }
}

// ------------------------------------------------------------------ convert: dq = scale * accumulator
// One CTA per 64-query block: 256 threads, each converting 8-element chunks of rows.
template <typename T, int D, bool VARLEN>
__global__ void __launch_bounds__(256) fmha_bwd_dq_kernel(const RowParams p) {
  const int bh = (int)blockIdx.y + (int)blockIdx.z * (int)gridDim.y;
  if (bh >= p.zh) return;
  const int h = bh % p.hq;
  const int zb = bh / p.hq;
  const int jb = blockIdx.x;
  int row_q0 = 0, len_q = p.sq;
  int64_t base = 0;
  if constexpr (VARLEN) {
    varlen_rows(p.cu_q, zb, p.total_q, row_q0, len_q);
    base = varlen_block_base(row_q0, zb);
  }
  if (jb * kBM >= len_q) return;
  const int64_t tile = (VARLEN ? (int64_t)h : (int64_t)bh) * p.tiles_per_head + base + jb;
  const float* src = p.dq_acc + tile * (kBM * D);
  constexpr int kChunks = kBM * D / 8;
  for (int i = threadIdx.x; i < kChunks; i += 256) {
    const int q = i / (D / 8), c = i % (D / 8);
    const int qi = jb * kBM + q;
    if (qi >= len_q) continue;
    const float4 a = *reinterpret_cast<const float4*>(src + q * D + c * 8);
    const float4 b = *reinterpret_cast<const float4*>(src + q * D + c * 8 + 4);
    T* dst;
    if constexpr (VARLEN)
      dst = reinterpret_cast<T*>(p.dq) + (int64_t)(row_q0 + qi) * p.dq_ss + (int64_t)h * p.dq_sh;
    else
      dst = reinterpret_cast<T*>(p.dq) + (int64_t)zb * p.dq_sz + (int64_t)h * p.dq_sh + (int64_t)qi * p.dq_ss;
    const float s = p.scale;
    *reinterpret_cast<uint4*>(dst + c * 8) =
        make_uint4(Cvt<T>::pack(a.x * s, a.y * s), Cvt<T>::pack(a.z * s, a.w * s), Cvt<T>::pack(b.x * s, b.y * s),
                   Cvt<T>::pack(b.z * s, b.w * s));
  }
}


// ------------------------------------------------------------------ host side
dim3 grid_of(int x, int64_t yz) {
  const unsigned y = (unsigned)(yz < 65535 ? yz : 65535);
  return dim3((unsigned)x, y, (unsigned)((yz + (int64_t)y - 1) / (int64_t)y));
}

bool make_map(CUtensorMap* m, int dtype, const void* base, int64_t z, int64_t h, int64_t s, int64_t d,
              int64_t sz, int64_t sh, int64_t ss, uint32_t rows) {
  uint64_t dims[4] = {(uint64_t)d, (uint64_t)s, (uint64_t)h, (uint64_t)z};
  uint64_t str[3] = {(uint64_t)ss * 2, (uint64_t)sh * 2, (uint64_t)sz * 2};
  uint32_t box[4] = {64, rows, 1, 1};
  return host::encode_tmap(m, dtype, 4, base, dims, str, box);
}

template <typename T, int D, bool VARLEN, bool EXTRA>
int launch_main(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                const Params& p, dim3 grid, cudaStream_t s) {
  auto kern = fmha_bwd_kernel<T, D, VARLEN, EXTRA>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<D>::kBytes);
    if (e != cudaSuccess) return host::cuda_check(e, "cudaFuncSetAttribute(fmha bwd)");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  kern<<<grid, kThreads, Layout<D>::kBytes, s>>>(tq, tk, tv, tdo, p);
  return host::cuda_check(cudaGetLastError(), "fmha bwd kernel launch");
}

template <typename T, int D, bool VARLEN>
int run_all(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
            const Params& p, const RowParams& rp, int q_blocks, int kv_tiles, bool extra, cudaStream_t s) {
  const dim3 rgrid = grid_of(q_blocks, rp.zh);
  if (q_blocks > 0) {
    fmha_bwd_prep_kernel<T, D, VARLEN><<<rgrid, 256, 0, s>>>(rp);
    int rc = host::cuda_check(cudaGetLastError(), "fmha bwd prep launch");
    if (rc) return rc;
  }
  if (kv_tiles > 0) {
    const dim3 g = grid_of(kv_tiles, p.zh_kv);
    int rc = extra ? launch_main<T, D, VARLEN, true>(tq, tk, tv, tdo, p, g, s)
                   : launch_main<T, D, VARLEN, false>(tq, tk, tv, tdo, p, g, s);
    if (rc) return rc;
  }
  if (q_blocks > 0) {
    fmha_bwd_dq_kernel<T, D, VARLEN><<<rgrid, 256, 0, s>>>(rp);
    return host::cuda_check(cudaGetLastError(), "fmha bwd dq launch");
  }
  return GKO_OK;
}

template <bool VARLEN>
int dispatch(int dtype, int d, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
             const CUtensorMap& tdo, const Params& p, const RowParams& rp, int q_blocks, int kv_tiles, bool extra,
             cudaStream_t s) {
  if (dtype == GKO_BF16)
    return d == 64 ? run_all<__nv_bfloat16, 64, VARLEN>(tq, tk, tv, tdo, p, rp, q_blocks, kv_tiles, extra, s)
                   : run_all<__nv_bfloat16, 128, VARLEN>(tq, tk, tv, tdo, p, rp, q_blocks, kv_tiles, extra, s);
  return d == 64 ? run_all<__half, 64, VARLEN>(tq, tk, tv, tdo, p, rp, q_blocks, kv_tiles, extra, s)
                 : run_all<__half, 128, VARLEN>(tq, tk, tv, tdo, p, rp, q_blocks, kv_tiles, extra, s);
}

int64_t workspace_tiles(int64_t batch, int64_t hq, int64_t sq_or_tq, int varlen) {
  const int64_t blocks = (sq_or_tq + kBM - 1) / kBM;
  return varlen ? hq * (blocks + batch + 1) : batch * hq * blocks;
}

int check_common(int dtype, int64_t hq, int64_t hkv, int64_t d, float scale, int window, float softcap) {
  using host::fail;
  if (dtype != GKO_F16 && dtype != GKO_BF16)
    return fail(GKO_ERR_UNSUPPORTED, "fmha backward supports float16 and bfloat16 only (dtype code %d)", dtype);
  if (d != 64 && d != 128)
    return fail(GKO_ERR_UNSUPPORTED, "fmha backward supports head dim 64 or 128, got %lld", (long long)d);
  if (hq <= 0 || hkv <= 0 || hq % hkv)
    return fail(GKO_ERR_INVALID, "query heads (%lld) must be a positive multiple of kv heads (%lld)",
                (long long)hq, (long long)hkv);
  if (window < 0) return fail(GKO_ERR_INVALID, "window must be >= 0");
  if (!(softcap >= 0.f)) return fail(GKO_ERR_INVALID, "softcap must be >= 0");
  if (!(scale == scale)) return fail(GKO_ERR_INVALID, "scale is NaN");
  return GKO_OK;
}

bool strides_ok(const int64_t* s, int n) {
  for (int i = 0; i < n; ++i)
    if (s[i] < 0 || s[i] % 8) return false;
  return true;
}

}  // namespace fmha_bwd
}  // namespace gko

using namespace gko;
using gko::host::fail;

extern "C" int64_t gko_fmha_bwd_workspace_size(int64_t batch, int64_t hq, int64_t sq_or_tq, int64_t d,
                                               int varlen) {
  if (batch < 0 || hq < 0 || sq_or_tq < 0 || (d != 64 && d != 128)) return -1;
  const int64_t tiles = fmha_bwd::workspace_tiles(batch, hq, sq_or_tq, varlen);
  return tiles * (fmha_bwd::kBM * d * 4 + 2 * fmha_bwd::kBM * 4);
}

extern "C" int gko_fmha_bwd(int dtype, int64_t z, int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int64_t d,
                            const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
                            const int64_t* vs, const void* bias, int bias_mode, int bias_dtype,
                            const int64_t* bs, int64_t bias_batch, const void* out, const int64_t* os,
                            const void* dout, const int64_t* dos, const float* lse, float scale, int causal,
                            int window, float softcap, void* dq, const int64_t* dqs, void* dk,
                            const int64_t* dks, void* dv, const int64_t* dvs, void* workspace,
                            int64_t workspace_bytes, unsigned int* status, void* stream) {
  int rc = fmha_bwd::check_common(dtype, hq, hkv, d, scale, window, softcap);
  if (rc) return rc;
  if (z < 0 || sq < 0 || sk < 0) return fail(GKO_ERR_INVALID, "negative attention size");
  if (z == 0 || (sq == 0 && sk == 0)) return GKO_OK;
  if (!q || !k || !v || !out || !dout || !lse || !dq || !dk || !dv || !qs || !ks || !vs || !os || !dos || !dqs ||
      !dks || !dvs)
    return fail(GKO_ERR_INVALID, "null pointer argument");
  const int64_t* all[8] = {qs, ks, vs, os, dos, dqs, dks, dvs};
  for (const int64_t* s : all) {
    if (s[3] != 1) return fail(GKO_ERR_UNSUPPORTED, "fmha backward needs unit stride along the head dim");
    if (!fmha_bwd::strides_ok(s, 3))
      return fail(GKO_ERR_UNSUPPORTED, "fmha backward needs non-negative strides that are multiples of 8 elements");
  }
  const void* ptrs[8] = {q, k, v, out, dout, dq, dk, dv};
  for (const void* ptr : ptrs)
    if (!host::aligned16(ptr)) return fail(GKO_ERR_UNSUPPORTED, "fmha backward needs 16-byte aligned tensors");
  if (sq > (1 << 30) || sk > (1 << 30) || z * hq >= (1ll << 31))
    return fail(GKO_ERR_UNSUPPORTED, "fmha backward sizes out of range");
  if (bias_mode != GKO_BIAS_NONE && bias_mode != GKO_BIAS_KEYPAD && bias_mode != GKO_BIAS_FULL)
    return fail(GKO_ERR_INVALID, "unknown bias mode %d", bias_mode);
  if (bias_mode != GKO_BIAS_NONE) {
    if (!bias || !bs) return fail(GKO_ERR_INVALID, "bias mode set but bias pointer is null");
    if (bias_dtype != GKO_F16 && bias_dtype != GKO_BF16 && bias_dtype != GKO_F32)
      return fail(GKO_ERR_INVALID, "unknown bias dtype %d", bias_dtype);
    if (bias_batch <= 0 || bias_batch > z || z % bias_batch)
      return fail(GKO_ERR_INVALID, "bias batch count %lld must divide the batch %lld", (long long)bias_batch,
                  (long long)z);
  }
  const int64_t need = gko_fmha_bwd_workspace_size(z, hq, sq, d, 0);
  if (!workspace || workspace_bytes < need || !host::aligned16(workspace))
    return fail(GKO_ERR_INVALID, "fmha backward needs a 16-byte aligned workspace of %lld bytes (got %lld)",
                (long long)need, (long long)workspace_bytes);
  const int64_t tiles = fmha_bwd::workspace_tiles(z, hq, sq, 0);
  float* ws = static_cast<float*>(workspace);
  CUtensorMap tq, tk, tv, tdo;
  const int64_t sqm = sq > 0 ? sq : 1, skm = sk > 0 ? sk : 1;
  if (!fmha_bwd::make_map(&tq, dtype, q, z, hq, sqm, d, qs[0], qs[1], qs[2], fmha_bwd::kBM) ||
      !fmha_bwd::make_map(&tdo, dtype, dout, z, hq, sqm, d, dos[0], dos[1], dos[2], fmha_bwd::kBM) ||
      !fmha_bwd::make_map(&tk, dtype, k, z, hkv, skm, d, ks[0], ks[1], ks[2], fmha_bwd::kBN) ||
      !fmha_bwd::make_map(&tv, dtype, v, z, hkv, skm, d, vs[0], vs[1], vs[2], fmha_bwd::kBN))
    return GKO_ERR_INVALID;
  fmha_bwd::Params p{};
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.group = (int)(hq / hkv);
  p.sq = (int)sq;
  p.sk = (int)sk;
  p.zh_kv = (int)(z * hkv);
  p.scale = scale;
  p.scale_log2 = scale * fmha_bwd::kLog2e;
  p.softcap = softcap;
  p.causal = causal ? 1 : 0;
  p.window = window;
  p.bias = bias;
  p.bias_mode = bias_mode;
  p.bias_dtype = bias_dtype;
  p.bias_z = bias_mode != GKO_BIAS_NONE ? (int)bias_batch : 1;
  if (bias_mode == GKO_BIAS_KEYPAD) {
    p.b_sz = bs[0];
    p.b_sk = bs[3];
  } else if (bias_mode == GKO_BIAS_FULL) {
    p.b_sz = bs[0];
    p.b_sh = bs[1];
    p.b_sq = bs[2];
    p.b_sk = bs[3];
  }
  p.dq_acc = ws;
  p.nl = ws + tiles * fmha_bwd::kBM * d;
  p.nd = p.nl + tiles * fmha_bwd::kBM;
  p.tiles_per_head = (sq + fmha_bwd::kBM - 1) / fmha_bwd::kBM;
  p.dk = dk;
  p.dk_sz = dks[0];
  p.dk_sh = dks[1];
  p.dk_ss = dks[2];
  p.dv = dv;
  p.dv_sz = dvs[0];
  p.dv_sh = dvs[1];
  p.dv_ss = dvs[2];
  p.status = status;
  fmha_bwd::RowParams rp{};
  rp.hq = (int)hq;
  rp.sq = (int)sq;
  rp.zh = (int)(z * hq);
  rp.o = out;
  rp.o_sz = os[0];
  rp.o_sh = os[1];
  rp.o_ss = os[2];
  rp.dout = dout;
  rp.do_sz = dos[0];
  rp.do_sh = dos[1];
  rp.do_ss = dos[2];
  rp.lse = lse;
  rp.lse_stride_h = sq;
  rp.dq_acc = p.dq_acc;
  rp.nl = const_cast<float*>(p.nl);
  rp.nd = const_cast<float*>(p.nd);
  rp.tiles_per_head = p.tiles_per_head;
  rp.dq = dq;
  rp.dq_sz = dqs[0];
  rp.dq_sh = dqs[1];
  rp.dq_ss = dqs[2];
  rp.scale = scale;
  const bool extra = bias_mode != GKO_BIAS_NONE || softcap > 0.f || window > 0;
  const int q_blocks = (int)((sq + fmha_bwd::kBM - 1) / fmha_bwd::kBM);
  const int kv_tiles = (int)((sk + fmha_bwd::kBN - 1) / fmha_bwd::kBN);
  return fmha_bwd::dispatch<false>(dtype, (int)d, tq, tk, tv, tdo, p, rp, q_blocks, kv_tiles, extra,
                                   reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gko_fmha_varlen_bwd(int dtype, int64_t b, int64_t hq, int64_t hkv, int64_t d, int64_t tq,
                                   int64_t tk, int64_t max_seqlen_q, int64_t max_seqlen_k, const void* q,
                                   int64_t q_st, int64_t q_sh, const void* k, int64_t k_st, int64_t k_sh,
                                   const void* v, int64_t v_st, int64_t v_sh, const void* out, int64_t o_st,
                                   int64_t o_sh, const void* dout, int64_t do_st, int64_t do_sh, const float* lse,
                                   const int32_t* cu_q, const int32_t* cu_k, float scale, int causal, int window,
                                   float softcap, void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st,
                                   int64_t dk_sh, void* dv, int64_t dv_st, int64_t dv_sh, void* workspace,
                                   int64_t workspace_bytes, unsigned int* status, void* stream) {
  int rc = fmha_bwd::check_common(dtype, hq, hkv, d, scale, window, softcap);
  if (rc) return rc;
  if (b < 0 || tq < 0 || tk < 0 || max_seqlen_q < 0 || max_seqlen_k < 0)
    return fail(GKO_ERR_INVALID, "negative size");
  if (b == 0 || (tq == 0 && tk == 0)) return GKO_OK;
  if (!q || !k || !v || !out || !dout || !lse || !cu_q || !cu_k || !dq || !dk || !dv)
    return fail(GKO_ERR_INVALID, "null pointer argument");
  const int64_t st[12] = {q_st, q_sh, k_st, k_sh, v_st, v_sh, o_st, o_sh, do_st, do_sh, dq_st, dq_sh};
  if (!fmha_bwd::strides_ok(st, 12) || !fmha_bwd::strides_ok(&dk_st, 1) || !fmha_bwd::strides_ok(&dk_sh, 1) ||
      !fmha_bwd::strides_ok(&dv_st, 1) || !fmha_bwd::strides_ok(&dv_sh, 1))
    return fail(GKO_ERR_UNSUPPORTED, "fmha backward needs token/head strides that are multiples of 8");
  const void* ptrs[8] = {q, k, v, out, dout, dq, dk, dv};
  for (const void* ptr : ptrs)
    if (!host::aligned16(ptr)) return fail(GKO_ERR_UNSUPPORTED, "fmha backward needs 16-byte aligned tensors");
  if (tq >= (1ll << 31) || tk >= (1ll << 31) || b * hq >= (1ll << 31))
    return fail(GKO_ERR_UNSUPPORTED, "too many tokens");
  const int64_t need = gko_fmha_bwd_workspace_size(b, hq, tq, d, 1);
  if (!workspace || workspace_bytes < need || !host::aligned16(workspace))
    return fail(GKO_ERR_INVALID, "fmha backward needs a 16-byte aligned workspace of %lld bytes (got %lld)",
                (long long)need, (long long)workspace_bytes);
  const int64_t tiles = fmha_bwd::workspace_tiles(b, hq, tq, 1);
  float* ws = static_cast<float*>(workspace);
  CUtensorMap mq, mk, mv, mdo;
  const int64_t tqm = tq > 0 ? tq : 1, tkm = tk > 0 ? tk : 1;
  if (!fmha_bwd::make_map(&mq, dtype, q, 1, hq, tqm, d, tqm * q_st, q_sh, q_st, fmha_bwd::kBM) ||
      !fmha_bwd::make_map(&mdo, dtype, dout, 1, hq, tqm, d, tqm * do_st, do_sh, do_st, fmha_bwd::kBM) ||
      !fmha_bwd::make_map(&mk, dtype, k, 1, hkv, tkm, d, tkm * k_st, k_sh, k_st, fmha_bwd::kBN) ||
      !fmha_bwd::make_map(&mv, dtype, v, 1, hkv, tkm, d, tkm * v_st, v_sh, v_st, fmha_bwd::kBN))
    return GKO_ERR_INVALID;
  fmha_bwd::Params p{};
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.group = (int)(hq / hkv);
  p.zh_kv = (int)(b * hkv);
  p.scale = scale;
  p.scale_log2 = scale * fmha_bwd::kLog2e;
  p.softcap = softcap;
  p.causal = causal ? 1 : 0;
  p.window = window;
  p.bias_mode = GKO_BIAS_NONE;
  p.bias_z = 1;
  p.dq_acc = ws;
  p.nl = ws + tiles * fmha_bwd::kBM * d;
  p.nd = p.nl + tiles * fmha_bwd::kBM;
  p.tiles_per_head = tiles / hq;
  p.dk = dk;
  p.dk_sh = dk_sh;
  p.dk_ss = dk_st;
  p.dv = dv;
  p.dv_sh = dv_sh;
  p.dv_ss = dv_st;
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  p.total_q = (int)tq;
  p.total_k = (int)tk;
  p.status = status;
  fmha_bwd::RowParams rp{};
  rp.hq = (int)hq;
  rp.zh = (int)(b * hq);
  rp.o = out;
  rp.o_sh = o_sh;
  rp.o_ss = o_st;
  rp.dout = dout;
  rp.do_sh = do_sh;
  rp.do_ss = do_st;
  rp.lse = lse;
  rp.lse_stride_h = tq;
  rp.dq_acc = p.dq_acc;
  rp.nl = const_cast<float*>(p.nl);
  rp.nd = const_cast<float*>(p.nd);
  rp.tiles_per_head = p.tiles_per_head;
  rp.dq = dq;
  rp.dq_sh = dq_sh;
  rp.dq_ss = dq_st;
  rp.scale = scale;
  rp.cu_q = cu_q;
  rp.total_q = (int)tq;
  const bool extra = softcap > 0.f || window > 0;
  const int q_blocks = (int)((max_seqlen_q + fmha_bwd::kBM - 1) / fmha_bwd::kBM);
  const int kv_tiles = (int)((max_seqlen_k + fmha_bwd::kBN - 1) / fmha_bwd::kBN);
  return fmha_bwd::dispatch<true>(dtype, (int)d, mq, mk, mv, mdo, p, rp, q_blocks, kv_tiles, extra,
                                  reinterpret_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ allocation-free variant
// gko_fmha_bwd_noalloc runs the same three kernels as gko_fmha_bwd, with the
// workspace taken from this fixed device array instead of the caller. The array
// is part of the library's device image, so every GPU that loads the library
// holds these 32 MiB until the process exits.
namespace {
constexpr int64_t kNoAllocScratchBytes = 32ll << 20;
static __device__ __align__(256) unsigned char g_fmha_bwd_scratch[kNoAllocScratchBytes];

// Device address of g_fmha_bwd_scratch on the current device. In host code the
// array's name only stands in for the symbol; the address kernels need comes from
// cudaGetSymbolAddress, looked up once per device (with that device current).
void* noalloc_scratch() {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    host::cuda_check(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    host::fail(GKO_ERR_UNSUPPORTED, "device index %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fmha_bwd_scratch);
    if (e != cudaSuccess || !p) {
      host::cuda_check(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "cudaGetSymbolAddress(fmha bwd scratch)");
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}
}  // namespace

extern "C" int gko_fmha_bwd_noalloc(int dtype, int64_t z, int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int64_t d,
                                    const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                                    const void* v, const int64_t* vs, const void* bias, int bias_mode,
                                    int bias_dtype, const int64_t* bs, int64_t bias_batch, const void* out,
                                    const int64_t* os, const void* dout, const int64_t* dos, const float* lse,
                                    float scale, int causal, int window, float softcap, void* dq,
                                    const int64_t* dqs, void* dk, const int64_t* dks, void* dv,
                                    const int64_t* dvs, unsigned int* status, void* stream) {
  // the same argument checks and empty-problem return as gko_fmha_bwd, before the scratch
  // size check and before the scratch address is looked up
  int rc = fmha_bwd::check_common(dtype, hq, hkv, d, scale, window, softcap);
  if (rc) return rc;
  if (z < 0 || sq < 0 || sk < 0) return fail(GKO_ERR_INVALID, "negative attention size");
  if (z == 0 || (sq == 0 && sk == 0)) return GKO_OK;
  const int64_t need = gko_fmha_bwd_workspace_size(z, hq, sq, d, 0);
  if (need < 0) return fail(GKO_ERR_INVALID, "fmha backward: bad sizes (z %lld, hq %lld, sq %lld, d %lld)",
                            (long long)z, (long long)hq, (long long)sq, (long long)d);
  if (need > kNoAllocScratchBytes)
    return fail(GKO_ERR_UNSUPPORTED,
                "gko_fmha_bwd_noalloc: this problem needs %lld bytes of scratch, more than the library's fixed "
                "%lld bytes (z * hq * ceil(sq / 64) must stay within %lld blocks at d = %lld); call gko_fmha_bwd "
                "with a caller-provided workspace instead",
                (long long)need, (long long)kNoAllocScratchBytes,
                (long long)(kNoAllocScratchBytes / (fmha_bwd::kBM * d * 4 + 2 * fmha_bwd::kBM * 4)), (long long)d);
  void* scratch = noalloc_scratch();
  if (!scratch) return GKO_ERR_CUDA;
  return gko_fmha_bwd(dtype, z, hq, hkv, sq, sk, d, q, qs, k, ks, v, vs, bias, bias_mode, bias_dtype, bs, bias_batch,
                      out, os, dout, dos, lse, scale, causal, window, softcap, dq, dqs, dk, dks, dv, dvs, scratch,
                      kNoAllocScratchBytes, status, stream);
}
