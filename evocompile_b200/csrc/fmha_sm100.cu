// Fused multi-head attention forward for sm_100a (gko::fused_sdpa_pair,
// gko::cutlass_fmha_pair, gko::fmha_varlen_fwd).
//
// One CTA computes a 256-row query block (two 128-row tiles Q0, Q1) of one
// (batch, head) against the key range the masks allow, in 128-key tiles:
//   warp 8     TMA producer: Q0/Q1 once, then K_j / V_j into a 2-stage ring
//   warp 9     MMA issuer + TMEM owner. Per key tile j and query tile t it issues
//              S_t = Q_t K_j^T into TMEM, then (once softmax has written P_t)
//              O_t += P_t V_j with P_t read from TMEM (the TS form of tcgen05.mma),
//              then S_t for tile j+1 — so the tensor core works on one query tile
//              while the other tile's softmax runs.
//   warps 0-3  softmax of Q0, warps 4-7 softmax of Q1: one thread per query row
//              reads S_t from TMEM, applies scale / bias / softcap / masks, keeps
//              the running max and sum, writes P_t (bf16/f16) back into the S_t
//              columns, rescales O_t in TMEM only when the running max grows by
//              more than 2^8, and at the end normalises O_t and writes out / lse.
// TMEM (512 columns): S0|P0 [0,128), S1|P1 [128,256), O0 [256,256+D), O1 [384,384+D).
// Registers: the CTA launches with 12 x 32 threads x 168 registers; the
// producer/MMA warpgroup (warps 8-11) drops to 72 registers per thread and the two
// softmax warpgroups rise to 216 (2 x 128 x 216 + 128 x 72 = 64512, the whole launch;
// at 56 the MMA issuer spilled).
// Semantics follow the reference Triton kernel _flash_fwd
// (eval/kernels/fused_sdpa.py:25-157): logits = scale * q.k (+ bias), then
// softcap, then masks (key padding, causal key <= query, |key - query| <= window);
// lse = max + ln(sum). GQA maps query head h to kv head h / (hq / hkv).
#include <type_traits>

#include "host_common.h"
#include "sm100_ptx.cuh"

namespace gko {
namespace fmha {

constexpr int kBM = 128;           // rows of one query tile
constexpr int kQTiles = 2;         // query tiles per CTA
constexpr int kBlockM = kBM * kQTiles;
constexpr int kBN = 128;           // keys per tile
constexpr int kThreads = 384;      // 2 x 4 softmax warps, producer, MMA, 2 idle
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kRegsSoftmax = 216;
constexpr uint32_t kRegsControl = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsControl <= 384 * 168, "register split exceeds the launch");
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.f;  // log2 units
// K tiles are double or triple buffered (V always double): the S MMA of the next key tile
// waits on K, so a deeper K ring hides more TMA latency when shared memory allows it.
#ifndef GKO_FMHA_K_STAGES
#define GKO_FMHA_K_STAGES 2
#endif
constexpr int kKStages = GKO_FMHA_K_STAGES;
// Wait for K(j+1) right before the first S MMA that reads it (1) or before the PV MMAs of
// tile j (0).
#ifndef GKO_FMHA_LATE_KWAIT
#define GKO_FMHA_LATE_KWAIT 1
#endif

struct Params {
  int hq, hkv, group;  // group = hq / hkv
  int sq, sk;          // dense: per-batch lengths; varlen: unused
  int q_tiles;         // 256-row query blocks along the query axis (grid.x)
  int zh;              // batch (or sequences) x query heads
  float scale, scale_log2, softcap;
  int causal, window;
  // bias (dense only)
  const void* bias;
  int bias_mode, bias_dtype, bias_z;  // batch index = z % bias_z
  int64_t b_sz, b_sh, b_sq, b_sk;
  // outputs
  void* out;
  int64_t o_sz, o_sh, o_ss;  // dense output element strides (z, h, s); d stride 1
  float* lse;
  int64_t lse_stride_h;  // dense: sq (rows of one head); varlen: total tokens
  const int* cu_q;
  const int* cu_k;
  int total_q;  // varlen: tq
  unsigned* status;
};

template <int D>
struct Layout {
  static constexpr uint32_t kChunk = 128 * 128;  // one [128 rows x 128 B] swizzle block
  static constexpr int kChunks = D / 64;
  static constexpr uint32_t kTile = kChunks * kChunk;  // 128 x D elements
  static constexpr uint32_t kQ = 0;                          // Q0, Q1
  static constexpr uint32_t kK0 = kQ + 2 * kTile;            // K stages
  static constexpr uint32_t kV0 = kK0 + kKStages * kTile;    // V stages 0, 1
  static constexpr uint32_t kMeta = kV0 + 2 * kTile;
  // at least 120 KB so that a single CTA (and its 512 TMEM columns) occupies an SM
  static constexpr uint32_t kBytes = (1024 + kMeta + 256) > 122880 ? (1024 + kMeta + 256) : 122880;
};

__device__ __forceinline__ float bias_value(const Params& p, int z, int h, int q, int k) {
  const int64_t off = (int64_t)(z % p.bias_z) * p.b_sz + (int64_t)h * p.b_sh + (int64_t)q * p.b_sq +
                      (int64_t)k * p.b_sk;
  if (p.bias_dtype == GKO_F32) return __ldg(reinterpret_cast<const float*>(p.bias) + off);
  if (p.bias_dtype == GKO_BF16)
    return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(p.bias) + off));
  return __half2float(__ldg(reinterpret_cast<const __half*>(p.bias) + off));
}

template <typename T, int D, bool VARLEN, bool EXTRA>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using L = Layout<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = make_idesc_f16(kBF16, kBM, kBN, false, false);
  constexpr uint32_t kIdescO = make_idesc_f16(kBF16, kBM, D, false, true);

  // ---------------------------------------------------------- block geometry
  // grid.x walks the query blocks of one (batch, head) — heaviest (causal) first — so
  // the CTAs running at the same time share that head's K/V in L2.
  const int bh = (int)blockIdx.y + (int)blockIdx.z * (int)gridDim.y;
  if (bh >= p.zh) return;
  const int h = bh % p.hq;
  const int zb = bh / p.hq;  // batch (dense) or sequence (varlen)
  const int qb = p.q_tiles - 1 - (int)blockIdx.x;
  const int m0 = qb * kBlockM;
  int len_q, len_k, row_q0, row_k0;
  if constexpr (VARLEN) {
    row_q0 = p.cu_q[zb];
    len_q = p.cu_q[zb + 1] - row_q0;
    row_k0 = p.cu_k[zb];
    len_k = p.cu_k[zb + 1] - row_k0;
  } else {
    row_q0 = 0;
    len_q = p.sq;
    row_k0 = 0;
    len_k = p.sk;
  }
  if (m0 >= len_q) return;  // uniform across the CTA, before any barrier or TMEM use
  const int hk = h / p.group;
  const int zc = VARLEN ? 0 : zb;  // tensor-map batch coordinate

  // key-tile range [lo_t, hi_t) of each query tile (empty when the tile is past the end)
  int lo_t[kQTiles], hi_t[kQTiles];
#pragma unroll
  for (int t = 0; t < kQTiles; ++t) {
    const int mt = m0 + t * kBM;
    int k_lo = 0, k_hi = len_k;
    if (p.causal) k_hi = min(k_hi, mt + kBM);
    if (p.window > 0) {
      k_lo = max(k_lo, mt - p.window);
      k_hi = min(k_hi, mt + kBM + p.window);
    }
    if (mt >= len_q || k_hi <= k_lo) {
      lo_t[t] = hi_t[t] = 0;
    } else {
      lo_t[t] = k_lo / kBN;
      hi_t[t] = (k_hi + kBN - 1) / kBN;
    }
  }
  int lo = 1 << 30, hi = 0;
#pragma unroll
  for (int t = 0; t < kQTiles; ++t)
    if (hi_t[t] > lo_t[t]) {
      lo = min(lo, lo_t[t]);
      hi = max(hi, hi_t[t]);
    }
  const int n_tiles = hi > lo ? hi - lo : 0;

  // ---------------------------------------------------------- shared memory
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  const uint32_t sb = raw_addr + pad;
  uint8_t* meta = smem_raw + pad + L::kMeta;
  const uint32_t smeta = sb + L::kMeta;
  const uint32_t bar_q = smeta;
  const uint32_t bar_kfull = smeta + 8;     // [kKStages <= 3]
  const uint32_t bar_kempty = smeta + 32;   // [kKStages <= 3]
  const uint32_t bar_vfull = smeta + 56;    // [2]
  const uint32_t bar_vempty = smeta + 72;   // [2]
  const uint32_t bar_sfull = smeta + 88;    // [2] per query tile
  // [2 query tiles][2 halves]: P is handed over in two halves; a barrier per half
  // completes once per key tile, so a waiter can never miss a phase.
  const uint32_t bar_pfull = smeta + 104;
  const uint32_t bar_ofinal = smeta + 136;  // [2] per query tile
  const uint32_t bar_drain = smeta + 152;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(meta + 160);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 164);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(bar_kfull + 8 * i, 1);
      mbar_init(bar_kempty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_vfull + 8 * i, 1);
      mbar_init(bar_vempty + 8 * i, 1);
      mbar_init(bar_sfull + 8 * i, 1);
      mbar_init(bar_pfull + 16 * i, 4);
      mbar_init(bar_pfull + 16 * i + 8, 4);
      mbar_init(bar_ofinal + 8 * i, 1);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Each role's code is dominated by its warpgroup's setmaxnreg (no join in between),
  // so the compiler allocates the softmax code against 216 registers.
  if (warp >= kProducerWarp) {
  setmaxnreg_dec<kRegsControl>();
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n_tiles > 0) {
      mbar_arrive_expect_tx(bar_q, kQTiles * L::kTile);
#pragma unroll
      for (int t = 0; t < kQTiles; ++t)
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(sb + L::kQ + t * L::kTile + c * L::kChunk, &tm_q, bar_q, c * 64,
                      row_q0 + m0 + t * kBM, h, zc);
      for (int u = 0; u < n_tiles; ++u) {
        const int st = u & 1;
        const uint32_t ph = (u >> 1) & 1;
        const int ks = u % kKStages;
        const uint32_t kph = (u / kKStages) & 1;
        const int krow = row_k0 + (lo + u) * kBN;
        if (!wait_bounded(bar_kempty + 8 * ks, kph ^ 1, abort_flag, p.status, kStatusTimeoutProducer))
          break;
        mbar_arrive_expect_tx(bar_kfull + 8 * ks, L::kTile);
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(sb + L::kK0 + ks * L::kTile + c * L::kChunk, &tm_k, bar_kfull + 8 * ks, c * 64,
                      krow, hk, zc);
        if (!wait_bounded(bar_vempty + 8 * st, ph ^ 1, abort_flag, p.status, kStatusTimeoutProducer))
          break;
        mbar_arrive_expect_tx(bar_vfull + 8 * st, L::kTile);
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(sb + L::kV0 + st * L::kTile + c * L::kChunk, &tm_v, bar_vfull + 8 * st, c * 64,
                      krow, hk, zc);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      bool ok = wait_bounded(bar_q, 0, abort_flag, p.status, kStatusTimeoutMma);
      auto issue_s = [&](int t, int u) {
        const uint32_t k_addr = sb + L::kK0 + (u % kKStages) * L::kTile;
        const uint32_t q_addr = sb + L::kQ + t * L::kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kChunk + (kk & 3) * 32;
          mma_f16_ss(tmem_base + t * kBN, make_sdesc_sw128(q_addr + off, 16, 1024),
                     make_sdesc_sw128(k_addr + off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar_sfull + 8 * t);
      };
      // O_t += P_t V_j over keys [64 * half, 64 * half + 64) of the tile
      auto issue_pv = [&](int t, int u, bool first, int half) {
        const int st = u & 1;
        const uint32_t v_addr = sb + L::kV0 + st * L::kTile;
        const uint32_t o_tmem = tmem_base + 256 + t * 128;
        const uint32_t p_tmem = tmem_base + t * kBN;
#pragma unroll
        for (int k4 = 0; k4 < kBN / 32; ++k4) {
          const int kk = half * (kBN / 32) + k4;
          mma_f16_ts(o_tmem, p_tmem + kk * 8, make_sdesc_sw128(v_addr + kk * 16 * 128, L::kChunk, 1024),
                     kIdescO, (!first || kk > 0) ? 1u : 0u);
        }
      };
      // prologue: S_t for the first key tile
      if (ok) ok = wait_bounded(bar_kfull, 0, abort_flag, p.status, kStatusTimeoutMma);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < kQTiles; ++t)
          if (lo >= lo_t[t] && lo < hi_t[t]) issue_s(t, 0);
        mma_commit(bar_kempty);
      }
      for (int u = 0; u < n_tiles && ok; ++u) {
        const int j = lo + u;
        const int st = u & 1;
        const uint32_t ph = (u >> 1) & 1;
        ok = wait_bounded(bar_vfull + 8 * st, ph, abort_flag, p.status, kStatusTimeoutMma);
        const bool next = (u + 1 < n_tiles);
        const int kn = (u + 1) % kKStages;
        const uint32_t knph = ((u + 1) / kKStages) & 1;
        bool k_ready = !next;
        if (!GKO_FMHA_LATE_KWAIT && ok && next) {
          ok = wait_bounded(bar_kfull + 8 * kn, knph, abort_flag, p.status, kStatusTimeoutMma);
          k_ready = true;
        }
        if (!ok) break;
#pragma unroll
        for (int t = 0; t < kQTiles && ok; ++t) {
          if (j >= lo_t[t] && j < hi_t[t]) {
            // softmax hands P over in two halves, one barrier each
#pragma unroll
            for (int half = 0; half < 2 && ok; ++half) {
              ok = wait_bounded(bar_pfull + 16 * t + 8 * half, (j - lo_t[t]) & 1, abort_flag, p.status,
                                kStatusTimeoutMma);
              if (!ok) break;
              tc_fence_after();
              issue_pv(t, u, j == lo_t[t], half);
            }
            if (!ok) break;
            if (j == hi_t[t] - 1) mma_commit(bar_ofinal + 8 * t);
          }
          if (next && j + 1 >= lo_t[t] && j + 1 < hi_t[t]) {
            if (!k_ready) {
              ok = wait_bounded(bar_kfull + 8 * kn, knph, abort_flag, p.status, kStatusTimeoutMma);
              if (!ok) break;
              tc_fence_after();
              k_ready = true;
            }
            issue_s(t, u + 1);
          }
        }
        if (!ok) break;
        if (next && !k_ready) {  // K(j+1) unused by both tiles: still consume its load before release
          ok = wait_bounded(bar_kfull + 8 * kn, knph, abort_flag, p.status, kStatusTimeoutMma);
          if (!ok) break;
        }
        mma_commit(bar_vempty + 8 * st);
        if (next) mma_commit(bar_kempty + 8 * kn);
      }
      if (*abort_flag) {
        mma_commit(bar_drain);
        wait_for(bar_drain, 0, p.status, kStatusTimeoutDrain);
      }
    }
  }
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax / epilogue
    const int t = warp >> 2;            // query tile of this warpgroup
    const int quarter = warp & 3;       // TMEM lane quarter
    const int r = quarter * 32 + lane;  // query row within the tile
    const int qi = m0 + t * kBM + r;    // query index within the sequence
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem_base + lane_off + t * kBN;
    const uint32_t o_tmem = tmem_base + lane_off + 256 + t * 128;
    const int jlo = t ? lo_t[1] : lo_t[0];
    const int jhi = t ? hi_t[1] : hi_t[0];
    const int mt = m0 + t * kBM;
    float m_run = -INFINITY;  // running max, log2 domain
    float l_run = 0.f;
    bool ok = true;
    for (int j = jlo; j < jhi; ++j) {
      const int i = j - jlo;
      const int kbase = j * kBN;
      if (!wait_bounded(bar_sfull + 8 * t, i & 1, abort_flag, p.status, kStatusTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kBN];
      {
        uint32_t su[kBN];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_ld32p(s_tmem + c * 32, su + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kBN; ++c) s[c] = __uint_as_float(su[c]);
      }
      // Row maximum. The plain path keeps raw scores (scale > 0 is folded into the
      // exponent FFMA below); the general path converts to log2-domain logits first.
      float kmul;  // multiplier taking s[] to the log2 domain
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
      if constexpr (EXTRA) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const int kj = kbase + c;
          float x = s[c] * p.scale;
          if (p.bias_mode != GKO_BIAS_NONE && kj < len_k && qi < len_q) x += bias_value(p, zb, h, qi, kj);
          if (p.softcap > 0.f) x = p.softcap * tanhf(fminf(fmaxf(x / p.softcap, -15.f), 15.f));
          bool keep = kj < len_k;
          if (p.causal) keep = keep && (kj <= qi);
          if (p.window > 0) keep = keep && (kj - qi <= p.window) && (qi - kj <= p.window);
          s[c] = keep ? x * kLog2e : -INFINITY;
        }
        kmul = 1.f;
      } else {
        const bool need_mask = (kbase + kBN > len_k) || (p.causal && kbase + kBN - 1 > mt);
        if (need_mask) {
          // keys kbase + c with c >= lim are masked (past the end, or after the query when causal)
          const int lim = min(len_k, p.causal ? qi + 1 : len_k) - kbase;
#pragma unroll
          for (int c = 0; c < kBN; ++c) s[c] = (c < lim) ? s[c] : -INFINITY;
        }
        kmul = p.scale_log2;
      }
#pragma unroll
      for (int c = 0; c < kBN; c += 8) {
        mx0 = max3f(mx0, s[c], s[c + 1]);
        mx1 = max3f(mx1, s[c + 2], s[c + 3]);
        mx2 = max3f(mx2, s[c + 4], s[c + 5]);
        mx3 = max3f(mx3, s[c + 6], s[c + 7]);
      }
      const float tmax = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * kmul;
      // lazy rescale: keep the old max unless the new one exceeds it by the threshold
      float m_new = m_run;
      float alpha = 1.f;
      if (tmax > m_run + kRescaleThreshold) {
        m_new = tmax;
        alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
      }
      // O_t is stable here: S_t(j) completing implies PV_t(j-1) (issued before it) completed.
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_tmem + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(o_tmem + c * 32, o);
        }
      }
      // P_t = 2^(kmul * s - m): one packed FFMA per pair, then MUFU.EX2. P (bf16/f16
      // pairs) goes into the first kBN/2 columns of the S_t region, 64 keys at a time.
      const float nm = (m_new == -INFINITY) ? 0.f : -m_new;
      const uint64_t k2 = f2pack(kmul, kmul), nm2 = f2pack(nm, nm);
      float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          float a, b;
          f2unpack(fma2(f2pack(s[half * 64 + 2 * c], s[half * 64 + 2 * c + 1]), k2, nm2), a, b);
          a = fast_exp2(a);
          b = fast_exp2(b);
          if (c & 1) {
            acc2 += a;
            acc3 += b;
          } else {
            acc0 += a;
            acc1 += b;
          }
          pk[c] = Cvt<T>::pack(a, b);
        }
        tmem_st32(s_tmem + half * 32, pk);
        // hand this half of P to the MMA warp
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_pfull + 16 * t + 8 * half);
      }
      const float rsum = (acc0 + acc1) + (acc2 + acc3);
      l_run = l_run * alpha + rsum;
      m_run = m_new;
    }

    // ---------------------------------------------------------- epilogue
    const bool has = jhi > jlo;
    if (ok && has) {
      ok = wait_bounded(bar_ofinal + 8 * t, 0, abort_flag, p.status, kStatusTimeoutSoftmax);
      tc_fence_after();
    }
    // varlen: rows outside [0, total_q) (cu_seqlens past the packed tokens) are never written
    const bool write = qi < len_q && (!VARLEN || (row_q0 >= 0 && row_q0 + qi < p.total_q));
    T* orow;
    if constexpr (VARLEN)
      orow = reinterpret_cast<T*>(p.out) + ((int64_t)(row_q0 + qi) * p.hq + h) * D;
    else
      orow = reinterpret_cast<T*>(p.out) + (int64_t)zb * p.o_sz + (int64_t)h * p.o_sh + (int64_t)qi * p.o_ss;
    const float inv = (l_run > 0.f) ? 1.f / l_run : 0.f;
    if (ok && has) {
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_tmem + c * 32, o);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          w[e] = Cvt<T>::pack(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
        if (write) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
    } else if (write) {
      uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
      for (int e = 0; e < D / 8; ++e) dst[e] = make_uint4(0, 0, 0, 0);
    }
    if (write) {
      const float lse = (l_run > 0.f) ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
      if constexpr (VARLEN)
        p.lse[(int64_t)h * p.lse_stride_h + row_q0 + qi] = lse;
      else
        p.lse[((int64_t)zb * p.hq + h) * p.lse_stride_h + qi] = lse;
    }
    tc_fence_before();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ host side
template <typename T, int D, bool VARLEN, bool EXTRA>
int launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
           dim3 grid, cudaStream_t s) {
  auto kern = fmha_fwd_kernel<T, D, VARLEN, EXTRA>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<D>::kBytes);
    if (e != cudaSuccess) return host::cuda_check(e, "cudaFuncSetAttribute(fmha)");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  kern<<<grid, kThreads, Layout<D>::kBytes, s>>>(tq, tk, tv, p);
  return host::cuda_check(cudaGetLastError(), "fmha kernel launch");
}

template <typename T, bool VARLEN>
int dispatch(int d, bool extra, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
             const Params& p, dim3 grid, cudaStream_t s) {
  if (d == 64)
    return extra ? launch<T, 64, VARLEN, true>(tq, tk, tv, p, grid, s)
                 : launch<T, 64, VARLEN, false>(tq, tk, tv, p, grid, s);
  return extra ? launch<T, 128, VARLEN, true>(tq, tk, tv, p, grid, s)
               : launch<T, 128, VARLEN, false>(tq, tk, tv, p, grid, s);
}

// Grid: query blocks along x, (batch, head) pairs along y (and z beyond 65535).
dim3 grid_of(int q_blocks, int zh) {
  const unsigned y = (unsigned)(zh < 65535 ? zh : 65535);
  return dim3((unsigned)q_blocks, y, (unsigned)((zh + (int)y - 1) / (int)y));
}

// 4-D tensor map over (d, s, h, z) for one operand; strides in elements for (z, h, s).
bool make_map(CUtensorMap* m, int dtype, const void* base, int64_t z, int64_t h, int64_t s, int64_t d,
              int64_t sz, int64_t sh, int64_t ss) {
  uint64_t dims[4] = {(uint64_t)d, (uint64_t)s, (uint64_t)h, (uint64_t)z};
  uint64_t str[3] = {(uint64_t)ss * 2, (uint64_t)sh * 2, (uint64_t)sz * 2};
  uint32_t box[4] = {64, 128, 1, 1};
  return host::encode_tmap(m, dtype, 4, base, dims, str, box);
}

int check_common(int dtype, int64_t hq, int64_t hkv, int64_t d, float scale, int window, float softcap) {
  using host::fail;
  if (dtype != GKO_F16 && dtype != GKO_BF16)
    return fail(GKO_ERR_UNSUPPORTED, "fmha supports float16 and bfloat16 only (dtype code %d)", dtype);
  if (d != 64 && d != 128)
    return fail(GKO_ERR_UNSUPPORTED, "fmha supports head dim 64 or 128, got %lld", (long long)d);
  if (hq <= 0 || hkv <= 0 || hq % hkv)
    return fail(GKO_ERR_INVALID, "query heads (%lld) must be a positive multiple of kv heads (%lld)",
                (long long)hq, (long long)hkv);
  if (window < 0) return fail(GKO_ERR_INVALID, "window must be >= 0");
  if (!(softcap >= 0.f)) return fail(GKO_ERR_INVALID, "softcap must be >= 0");
  if (!(scale == scale)) return fail(GKO_ERR_INVALID, "scale is NaN");
  return GKO_OK;
}

}  // namespace fmha
}  // namespace gko

using namespace gko;
using gko::host::fail;

extern "C" int gko_fmha_fwd(int dtype, int64_t z, int64_t hq, int64_t hkv, int64_t sq, int64_t sk,
                            int64_t d, const void* q, const int64_t* qs, const void* k,
                            const int64_t* ks, const void* v, const int64_t* vs, const void* bias,
                            int bias_mode, int bias_dtype, const int64_t* bs, int64_t bias_batch,
                            const int64_t* os, float scale,
                            int causal, int window, float softcap, void* out, float* lse,
                            unsigned int* status, void* stream) {
  int rc = fmha::check_common(dtype, hq, hkv, d, scale, window, softcap);
  if (rc) return rc;
  if (z < 0 || sq < 0 || sk < 0) return fail(GKO_ERR_INVALID, "negative attention size");
  if (z == 0 || sq == 0) return GKO_OK;
  if (!q || !k || !v || !out || !lse || !qs || !ks || !vs)
    return fail(GKO_ERR_INVALID, "null pointer argument");
  if (qs[3] != 1 || ks[3] != 1 || vs[3] != 1)
    return fail(GKO_ERR_UNSUPPORTED, "fmha needs unit stride along the head dim");
  for (int i = 0; i < 3; ++i)
    if (qs[i] % 8 || ks[i] % 8 || vs[i] % 8 || qs[i] < 0 || ks[i] < 0 || vs[i] < 0)
      return fail(GKO_ERR_UNSUPPORTED,
                  "fmha needs non-negative q/k/v strides that are multiples of 8 elements");
  if (!host::aligned16(q) || !host::aligned16(k) || !host::aligned16(v) || !host::aligned16(out))
    return fail(GKO_ERR_UNSUPPORTED, "fmha needs 16-byte aligned q, k, v, out");
  if (sq > (1 << 30) || sk > (1 << 30) || z * hq >= (1ll << 31))
    return fail(GKO_ERR_UNSUPPORTED, "fmha sizes out of range");
  if (bias_mode != GKO_BIAS_NONE && bias_mode != GKO_BIAS_KEYPAD && bias_mode != GKO_BIAS_FULL)
    return fail(GKO_ERR_INVALID, "unknown bias mode %d", bias_mode);
  if (bias_mode != GKO_BIAS_NONE) {
    if (!bias || !bs) return fail(GKO_ERR_INVALID, "bias mode set but bias pointer is null");
    if (bias_dtype != GKO_F16 && bias_dtype != GKO_BF16 && bias_dtype != GKO_F32)
      return fail(GKO_ERR_INVALID, "unknown bias dtype %d", bias_dtype);
  }
  CUtensorMap tq, tk, tv;
  if (!fmha::make_map(&tq, dtype, q, z, hq, sq, d, qs[0], qs[1], qs[2]) ||
      !fmha::make_map(&tk, dtype, k, z, hkv, sk > 0 ? sk : 1, d, ks[0], ks[1], ks[2]) ||
      !fmha::make_map(&tv, dtype, v, z, hkv, sk > 0 ? sk : 1, d, vs[0], vs[1], vs[2]))
    return GKO_ERR_INVALID;
  fmha::Params p{};
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.group = (int)(hq / hkv);
  p.sq = (int)sq;
  p.sk = (int)sk;
  p.q_tiles = (int)((sq + fmha::kBlockM - 1) / fmha::kBlockM);
  p.scale = scale;
  p.scale_log2 = scale * fmha::kLog2e;
  p.softcap = softcap;
  p.causal = causal ? 1 : 0;
  p.window = window;
  p.bias = bias;
  p.bias_mode = bias_mode;
  p.bias_dtype = bias_dtype;
  p.bias_z = 1;
  if (bias_mode == GKO_BIAS_KEYPAD) {
    p.b_sz = bs[0];
    p.b_sh = 0;
    p.b_sq = 0;
    p.b_sk = bs[3];
  } else if (bias_mode == GKO_BIAS_FULL) {
    p.b_sz = bs[0];
    p.b_sh = bs[1];
    p.b_sq = bs[2];
    p.b_sk = bs[3];
  }
  if (bias_mode != GKO_BIAS_NONE) {
    if (bias_batch <= 0 || bias_batch > z || z % bias_batch)
      return fail(GKO_ERR_INVALID, "bias batch count %lld must divide the batch %lld",
                  (long long)bias_batch, (long long)z);
    p.bias_z = (int)bias_batch;
  }
  p.out = out;
  if (os) {
    if (os[3] != 1 || os[0] % 8 || os[1] % 8 || os[2] % 8 || os[0] < 0 || os[1] < 0 || os[2] < 0)
      return fail(GKO_ERR_UNSUPPORTED, "fmha output needs unit d stride and other strides multiples of 8");
    p.o_sz = os[0];
    p.o_sh = os[1];
    p.o_ss = os[2];
  } else {
    p.o_ss = d;
    p.o_sh = sq * d;
    p.o_sz = hq * sq * d;
  }
  p.lse = lse;
  p.lse_stride_h = sq;
  p.status = status;
  const bool extra = bias_mode != GKO_BIAS_NONE || softcap > 0.f || window > 0;
  p.zh = (int)(z * hq);
  const dim3 grid = fmha::grid_of(p.q_tiles, p.zh);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == GKO_BF16) return fmha::dispatch<__nv_bfloat16, false>((int)d, extra, tq, tk, tv, p, grid, s);
  return fmha::dispatch<__half, false>((int)d, extra, tq, tk, tv, p, grid, s);
}

extern "C" int gko_fmha_varlen_fwd(int dtype, int64_t b, int64_t hq, int64_t hkv, int64_t d,
                                   int64_t tq, int64_t tk, int64_t max_seqlen_q, const void* q,
                                   int64_t q_st, int64_t q_sh, const void* k, int64_t k_st,
                                   int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh,
                                   const int32_t* cu_q, const int32_t* cu_k, float scale, int causal,
                                   int window, float softcap, void* out, float* lse,
                                   unsigned int* status, void* stream) {
  int rc = fmha::check_common(dtype, hq, hkv, d, scale, window, softcap);
  if (rc) return rc;
  if (b < 0 || tq < 0 || tk < 0 || max_seqlen_q < 0) return fail(GKO_ERR_INVALID, "negative size");
  if (b == 0 || tq == 0 || max_seqlen_q == 0) return GKO_OK;
  if (!q || !k || !v || !out || !lse || !cu_q || !cu_k)
    return fail(GKO_ERR_INVALID, "null pointer argument");
  if (q_st % 8 || q_sh % 8 || k_st % 8 || k_sh % 8 || v_st % 8 || v_sh % 8)
    return fail(GKO_ERR_UNSUPPORTED, "fmha needs token/head strides that are multiples of 8");
  if (!host::aligned16(q) || !host::aligned16(k) || !host::aligned16(v) || !host::aligned16(out))
    return fail(GKO_ERR_UNSUPPORTED, "fmha needs 16-byte aligned q, k, v, out");
  if (tq >= (1ll << 31) || tk >= (1ll << 31) || b * hq >= (1ll << 31))
    return fail(GKO_ERR_UNSUPPORTED, "too many tokens or (sequence, head) pairs");
  CUtensorMap mq, mk, mv;
  if (!fmha::make_map(&mq, dtype, q, 1, hq, tq, d, tq * q_st, q_sh, q_st) ||
      !fmha::make_map(&mk, dtype, k, 1, hkv, tk > 0 ? tk : 1, d, tk * k_st, k_sh, k_st) ||
      !fmha::make_map(&mv, dtype, v, 1, hkv, tk > 0 ? tk : 1, d, tk * v_st, v_sh, v_st))
    return GKO_ERR_INVALID;
  fmha::Params p{};
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.group = (int)(hq / hkv);
  p.q_tiles = (int)((max_seqlen_q + fmha::kBlockM - 1) / fmha::kBlockM);
  p.scale = scale;
  p.scale_log2 = scale * fmha::kLog2e;
  p.softcap = softcap;
  p.causal = causal ? 1 : 0;
  p.window = window;
  p.bias_mode = GKO_BIAS_NONE;
  p.bias_z = 1;
  p.out = out;
  p.lse = lse;
  p.lse_stride_h = tq;
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  p.total_q = (int)tq;
  p.status = status;
  const bool extra = softcap > 0.f || window > 0;
  p.zh = (int)(b * hq);
  const dim3 grid = fmha::grid_of(p.q_tiles, p.zh);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == GKO_BF16) return fmha::dispatch<__nv_bfloat16, true>((int)d, extra, mq, mk, mv, p, grid, s);
  return fmha::dispatch<__half, true>((int)d, extra, mq, mk, mv, p, grid, s);
}
