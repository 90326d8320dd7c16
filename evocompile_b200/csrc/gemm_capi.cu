// C-ABI entry points for the fused GEMM operators (gko_addmm_act, gko_linear_swiglu).
#include "gemm_f32.cuh"
#include "gemm_sm100.cuh"
#include <atomic>
#include <cmath>

#include "host_common.h"

using namespace gko;
using gko::host::fail;

namespace {

// Upper bound on the CTAs (SMs) a tensor-core GEMM launch occupies; 0 = every SM. Set through
// gko_set_gemm_ctas so that a collective running on another stream keeps SMs of its own.
std::atomic<int> g_gemm_ctas{0};

int gemm_grid_limit() {
  const int sms = host::sm_count();
  const int lim = g_gemm_ctas.load(std::memory_order_relaxed);
  return (lim > 0 && lim < sms) ? lim : sms;
}

int bias_kind_of(const void* bias, int bias_dtype) {
  if (!bias) return kBiasNone;
  switch (bias_dtype) {
    case GKO_F16: return kBiasF16;
    case GKO_BF16: return kBiasBF16;
    case GKO_F32: return kBiasF32;
    default: return -1;
  }
}

template <typename T, int EPI, bool B_MN, bool A_MN = false>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& tx0,
              const CUtensorMap& tx1, const GemmParams& p, cudaStream_t stream) {
  auto kern = gemm::gemm_kernel<T, EPI, B_MN, A_MN>;
  static bool configured[64] = {false};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemm::kSmemBytes);
    if (e != cudaSuccess) return host::cuda_check(e, "cudaFuncSetAttribute(gemm)");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int limit = gemm_grid_limit();
  const int grid = p.num_tiles < limit ? p.num_tiles : limit;
  kern<<<grid, gemm::kThreads, gemm::kSmemBytes, stream>>>(ta, tb, td, tx0, tx1, p);
  return host::cuda_check(cudaGetLastError(), "gemm kernel launch");
}

template <typename T, int EPI, bool B_MN>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                const GemmParams& p, cudaStream_t stream) {
  auto kern = gemm::gemm_pair_kernel<T, EPI, B_MN>;
  static bool configured[64] = {false};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemm::kPairSmemBytes);
    if (e != cudaSuccess) return host::cuda_check(e, "cudaFuncSetAttribute(gemm pair)");
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int pairs = gemm_grid_limit() / 2;
  const int clusters = p.num_tiles < pairs ? p.num_tiles : pairs;
  kern<<<2 * clusters, gemm::kThreads, gemm::kPairSmemBytes, stream>>>(ta, tb, td, p);
  return host::cuda_check(cudaGetLastError(), "gemm pair kernel launch");
}

template <typename T>
int dispatch_pair(int epi, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                  const CUtensorMap& td, const GemmParams& p, cudaStream_t s) {
  if (!b_mn) {
    switch (epi) {
      case kEpiNone: return launch_pair<T, kEpiNone, false>(ta, tb, td, p, s);
      case kEpiGelu: return launch_pair<T, kEpiGelu, false>(ta, tb, td, p, s);
      case kEpiRelu: return launch_pair<T, kEpiRelu, false>(ta, tb, td, p, s);
      default: return launch_pair<T, kEpiSwiglu, false>(ta, tb, td, p, s);
    }
  }
  switch (epi) {
    case kEpiNone: return launch_pair<T, kEpiNone, true>(ta, tb, td, p, s);
    case kEpiGelu: return launch_pair<T, kEpiGelu, true>(ta, tb, td, p, s);
    case kEpiRelu: return launch_pair<T, kEpiRelu, true>(ta, tb, td, p, s);
    default: return launch_pair<T, kEpiSwiglu, true>(ta, tb, td, p, s);
  }
}

template <typename T>
int dispatch_tc(int epi, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                const CUtensorMap& td, const CUtensorMap& tx0, const CUtensorMap& tx1, const GemmParams& p,
                cudaStream_t s, bool a_mn = false) {
  if (a_mn)  // MN-major A: plain epilogue only (checked by the caller)
    return b_mn ? launch_tc<T, kEpiNone, true, true>(ta, tb, td, tx0, tx1, p, s)
                : launch_tc<T, kEpiNone, false, true>(ta, tb, td, tx0, tx1, p, s);
  if (!b_mn) {
    switch (epi) {
      case kEpiAllReduce: return launch_tc<T, kEpiAllReduce, false>(ta, tb, td, tx0, tx1, p, s);
      case kEpiNone: return launch_tc<T, kEpiNone, false>(ta, tb, td, tx0, tx1, p, s);
      case kEpiGelu: return launch_tc<T, kEpiGelu, false>(ta, tb, td, tx0, tx1, p, s);
      case kEpiRelu: return launch_tc<T, kEpiRelu, false>(ta, tb, td, tx0, tx1, p, s);
      default: return launch_tc<T, kEpiSwiglu, false>(ta, tb, td, tx0, tx1, p, s);
    }
  }
  switch (epi) {
    case kEpiNone: return launch_tc<T, kEpiNone, true>(ta, tb, td, tx0, tx1, p, s);
    case kEpiGelu: return launch_tc<T, kEpiGelu, true>(ta, tb, td, tx0, tx1, p, s);
    case kEpiRelu: return launch_tc<T, kEpiRelu, true>(ta, tb, td, tx0, tx1, p, s);
    default: return launch_tc<T, kEpiSwiglu, true>(ta, tb, td, tx0, tx1, p, s);
  }
}

// Tensor-core path. A: [M, K] row stride lda. B storage: K-major [nb_rows, K] row stride ldb
// (b_mn = false) or MN-major [K, nb_cols] row stride ldb (b_mn = true), where the logical
// B rows (output columns, SwiGLU: gate then up) number nb_total. D: [M, N_out] row stride ldd.
int run_tc(int dtype, int epi, int64_t M, int64_t N_out, int64_t K, int64_t nb_total,
           int64_t up_offset, const void* a, int64_t lda, const void* b, int64_t ldb, bool b_mn,
           const void* bias, int bias_kind, void* d, int64_t ldd, unsigned* status,
           cudaStream_t stream, void* red_mc = nullptr, void* const* red_peers = nullptr,
           int red_world = 0, void* aux = nullptr, int64_t aux_ld = 0, const void* resid = nullptr,
           int64_t resid_ld = 0, const float* row_scale = nullptr, bool a_mn = false, int rope_cols = 0,
           int rope_seq = 0, float rope_log2_theta = 0.f) {
  if (rope_cols > 0 && (epi != kEpiNone || bias || aux || resid || red_world || rope_cols % 128 || rope_seq <= 0 ||
                        rope_cols > N_out))
    return fail(GKO_ERR_UNSUPPORTED, "RoPE in the GEMM epilogue needs the plain epilogue (no bias, residual or "
                "pre-activation output), whole 128-column heads and a positive sequence length");
  if (a_mn && (epi != kEpiNone || aux || resid || row_scale || red_world))
    return fail(GKO_ERR_UNSUPPORTED, "a transposed (MN-major) mat1 is supported with the plain epilogue only");
  if (resid && (!host::aligned16(resid) || resid_ld % 8))
    return fail(GKO_ERR_UNSUPPORTED, "the residual needs a 16-byte aligned base and a row stride that is a "
                "multiple of 8");
  if (!host::aligned16(a) || !host::aligned16(b) || !host::aligned16(d) || (aux && !host::aligned16(aux)) ||
      (bias && !host::aligned16(bias)))
    return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs 16-byte aligned operand and bias bases");
  if (aux && aux_ld % 8)
    return fail(GKO_ERR_UNSUPPORTED, "the pre-activation output needs a row stride that is a multiple of 8");
  if (lda % 8 || ldb % 8 || ldd % 8)
    return fail(GKO_ERR_UNSUPPORTED,
                "tensor-core GEMM needs row strides that are multiples of 8 elements "
                "(lda=%lld ldb=%lld ldd=%lld)",
                (long long)lda, (long long)ldb, (long long)ldd);
  // K is a row count (no alignment rule) only when both operands are MN-major
  if ((K % 8 && !(a_mn && b_mn)) || N_out % 8)
    return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs K %% 8 == 0 and N %% 8 == 0 "
                "(K=%lld N=%lld)", (long long)K, (long long)N_out);
  if (b_mn && epi == kEpiSwiglu && up_offset % 8)
    return fail(GKO_ERR_UNSUPPORTED, "transposed SwiGLU weight needs h %% 8 == 0");
  if (M >= (1ll << 31) || N_out >= (1ll << 31) || K >= (1ll << 31))
    return fail(GKO_ERR_UNSUPPORTED, "GEMM dimensions must be < 2^31");
  const int esz = 2;
  CUtensorMap ta, tb, td;
  if (!a_mn) {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    uint64_t str[1] = {(uint64_t)(lda * esz)};
    uint32_t box[2] = {64, 128};
    if (!host::encode_tmap(&ta, dtype, 2, a, dims, str, box)) return GKO_ERR_INVALID;
  } else {
    // A stored [K, M] row-major (row stride lda): 64 M-columns x 64 K-rows per box
    uint64_t dims[2] = {(uint64_t)M, (uint64_t)K};
    uint64_t str[1] = {(uint64_t)(lda * esz)};
    uint32_t box[2] = {64, 64};
    if (!host::encode_tmap(&ta, dtype, 2, a, dims, str, box)) return GKO_ERR_INVALID;
  }
  if (!b_mn) {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)nb_total};
    uint64_t str[1] = {(uint64_t)(ldb * esz)};
    uint32_t box[2] = {64, 128};
    if (!host::encode_tmap(&tb, dtype, 2, b, dims, str, box)) return GKO_ERR_INVALID;
  } else {
    uint64_t dims[2] = {(uint64_t)nb_total, (uint64_t)K};
    uint64_t str[1] = {(uint64_t)(ldb * esz)};
    uint32_t box[2] = {64, 64};
    if (!host::encode_tmap(&tb, dtype, 2, b, dims, str, box)) return GKO_ERR_INVALID;
  }
  {
    uint64_t dims[2] = {(uint64_t)N_out, (uint64_t)M};
    uint64_t str[1] = {(uint64_t)(ldd * esz)};
    uint32_t box[2] = {64, 32};
    if (!host::encode_tmap(&td, dtype, 2, d, dims, str, box)) return GKO_ERR_INVALID;
  }
  // the pre-activation output, stored by TMA like D: [M, N_out] at aux (for SwiGLU the gate
  // columns) and, for SwiGLU, [M, N_out] at aux + N_out (the up columns; 16-byte aligned since
  // N_out % 8 == 0). Two views keep a ragged last gate chunk from spilling into the up columns.
  CUtensorMap tx0 = td, tx1 = td;
  if (aux) {
    uint64_t dims[2] = {(uint64_t)N_out, (uint64_t)M};
    uint64_t str[1] = {(uint64_t)(aux_ld * esz)};
    uint32_t box[2] = {64, 32};
    if (!host::encode_tmap(&tx0, dtype, 2, aux, dims, str, box)) return GKO_ERR_INVALID;
    if (epi == kEpiSwiglu &&
        !host::encode_tmap(&tx1, dtype, 2, static_cast<const uint8_t*>(aux) + N_out * esz, dims, str, box))
      return GKO_ERR_INVALID;
  }
  GemmParams p{};
  p.M = (int)M;
  p.N_out = (int)N_out;
  p.K = (int)K;
  p.up_offset = (int)up_offset;
  // CTA pairs (256-row tiles, cta_group::2) for M >= GKO_GEMM_PAIR_MIN_M. Off by default:
  // on B200 the single-CTA kernel measured ~5% higher tensor-pipe utilisation on the
  // Llama-3-8B MLP shapes (86% vs 79.5% active), so the pair path is kept for tuning only.
#ifndef GKO_GEMM_PAIR_MIN_M
#define GKO_GEMM_PAIR_MIN_M 0x7fffffff
#endif
  const bool pair = M >= GKO_GEMM_PAIR_MIN_M && epi != kEpiAllReduce && !aux && !resid && !row_scale && !a_mn;
  const int block_m = pair ? 2 * gemm::kBM : gemm::kBM;
  p.m_blocks = (int)((M + block_m - 1) / block_m);
  const int bn = gemm::block_n_out(epi);
  p.n_blocks = (int)((N_out + bn - 1) / bn);
  p.num_tiles = p.m_blocks * p.n_blocks;
  p.k_blocks = (int)((K + gemm::kBK - 1) / gemm::kBK);
  {
    // Raster: the operand a group of tiles shares (an A row-block group, or a B column-block
    // group) is sized to stay resident in L2 next to the streamed operand and the output
    // (loaded evict-last; the rest evict-first); pick the grouping axis that minimises the
    // estimated DRAM reads of the streamed operand. For long K the whole-panel budget leaves
    // groups of a few blocks, so a group is never narrower than the side of a byte-square
    // wave of concurrently running tiles (one per SM): sqrt(SMs * 256 / 128) A row-blocks or
    // sqrt(SMs * 128 / 256) B column-blocks (measured +6..17% on K = 28672, neutral at K <= 8192).
#ifndef GKO_GEMM_L2_GROUP_MB
// measured on B200 (sustained, power-capped): 48 MB gave the Llama-3-70B gate/up (16384 x 57344 x
// 8192) 12.37 ms against 12.79 at 32 MB and 14.3 at 64 MB (the group no longer stays in the 126 MB
// L2 next to the streamed operand); the 8B MLP and the 70B down / QKV shapes moved by under 2 %
#define GKO_GEMM_L2_GROUP_MB 48
#endif
    const double budget = GKO_GEMM_L2_GROUP_MB * 1024.0 * 1024.0;
    const double a_bytes = (double)M * K * esz, b_bytes = (double)nb_total * K * esz;
    const double a_blk = (double)block_m * K * esz, b_blk = (double)gemm::kMmaN * K * esz;
    const double sms = (double)host::sm_count();
    const int gm_wave = (int)(sqrt(sms * gemm::kMmaN / block_m) + 0.5);
    const int gn_wave = (int)(sqrt(sms * block_m / gemm::kMmaN) + 0.5);
    int gm = (int)(budget / a_blk), gn = (int)(budget / b_blk);
    gm = gm < gm_wave ? gm_wave : gm;
    gn = gn < gn_wave ? gn_wave : gn;
    gm = gm < 1 ? 1 : (gm > p.m_blocks ? p.m_blocks : gm);
    gn = gn < 1 ? 1 : (gn > p.n_blocks ? p.n_blocks : gn);
    const double t_m = a_bytes + b_bytes * (double)((p.m_blocks + gm - 1) / gm);
    const double t_n = b_bytes + a_bytes * (double)((p.n_blocks + gn - 1) / gn);
    p.raster_n = t_n < t_m ? 1 : 0;
    p.group = p.raster_n ? gn : gm;
  }
  p.bias = bias;
  p.bias_kind = bias_kind;
  p.status = status;
  p.red_mc = red_mc;
  p.red_peers = red_peers;
  p.red_world = red_world;
  p.red_ld = ldd;
  p.aux = aux;
  p.aux_ld = aux_ld;
  p.resid = resid;
  p.resid_ld = resid_ld;
  p.row_scale = row_scale;
  p.rope_cols = rope_cols;
  p.rope_seq = rope_seq;
  p.rope_log2_theta = rope_log2_theta;
  if (p.num_tiles == 0) return GKO_OK;
  if (pair) {
    if (dtype == GKO_BF16) return dispatch_pair<__nv_bfloat16>(epi, b_mn, ta, tb, td, p, stream);
    return dispatch_pair<__half>(epi, b_mn, ta, tb, td, p, stream);
  }
  if (dtype == GKO_BF16) return dispatch_tc<__nv_bfloat16>(epi, b_mn, ta, tb, td, tx0, tx1, p, stream, a_mn);
  return dispatch_tc<__half>(epi, b_mn, ta, tb, td, tx0, tx1, p, stream, a_mn);
}

int run_f32(int epi, int64_t M, int64_t N_out, int64_t K, int64_t up_offset, const float* a,
            int64_t sam, int64_t sak, const float* b, int64_t sbk, int64_t sbn, const void* bias,
            int bias_kind, float* d, int64_t ldd, unsigned* status, cudaStream_t stream) {
  if (M >= (1ll << 31) || N_out >= (1ll << 31) || K >= (1ll << 31))
    return fail(GKO_ERR_UNSUPPORTED, "GEMM dimensions must be < 2^31");
  GemmParams p{};
  p.M = (int)M;
  p.N_out = (int)N_out;
  p.K = (int)K;
  p.up_offset = (int)up_offset;
  p.bias = bias;
  p.bias_kind = bias_kind;
  p.status = status;
  dim3 grid((unsigned)((N_out + 63) / 64), (unsigned)((M + 63) / 64));
  if (grid.x == 0 || grid.y == 0) return GKO_OK;
  if (grid.y > 65535) return fail(GKO_ERR_UNSUPPORTED, "fp32 GEMM supports M < 4194304");
  switch (epi) {
    case kEpiNone:
      gemm_f32::kernel<kEpiNone><<<grid, 256, 0, stream>>>(a, sam, sak, b, sbk, sbn, d, ldd, p);
      break;
    case kEpiGelu:
      gemm_f32::kernel<kEpiGelu><<<grid, 256, 0, stream>>>(a, sam, sak, b, sbk, sbn, d, ldd, p);
      break;
    case kEpiRelu:
      gemm_f32::kernel<kEpiRelu><<<grid, 256, 0, stream>>>(a, sam, sak, b, sbk, sbn, d, ldd, p);
      break;
    default:
      gemm_f32::kernel<kEpiSwiglu><<<grid, 256, 0, stream>>>(a, sam, sak, b, sbk, sbn, d, ldd, p);
      break;
  }
  return host::cuda_check(cudaGetLastError(), "fp32 gemm kernel launch");
}

}  // namespace

extern "C" int gko_addmm_act(int dtype, int act, int64_t m, int64_t n, int64_t k, const void* a,
                             int64_t a_sm, int64_t a_sk, const void* b, int64_t b_sk,
                             int64_t b_sn, const void* bias, int bias_dtype, void* d, int64_t ldd,
                             unsigned int* status, void* stream) {
  if (host::dtype_size(dtype) == 0) return fail(GKO_ERR_INVALID, "unknown dtype code %d", dtype);
  if (act != GKO_ACT_NONE && act != GKO_ACT_GELU && act != GKO_ACT_RELU)
    return fail(GKO_ERR_INVALID, "unknown activation code %d", act);
  if (m < 0 || n < 0 || k < 0) return fail(GKO_ERR_INVALID, "negative GEMM size");
  if (m == 0 || n == 0) return GKO_OK;  // empty output: nothing is read or written
  if (!d || (k && (!a || !b))) return fail(GKO_ERR_INVALID, "null operand pointer");
  const int bk = bias_kind_of(bias, bias_dtype);
  if (bk < 0) return fail(GKO_ERR_INVALID, "unknown bias dtype code %d", bias_dtype);
  const int epi = act == GKO_ACT_GELU ? kEpiGelu : act == GKO_ACT_RELU ? kEpiRelu : kEpiNone;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (m == 0 || n == 0) return GKO_OK;
  if (dtype == GKO_F32)
    return run_f32(epi, m, n, k, 0, static_cast<const float*>(a), a_sm, a_sk,
                   static_cast<const float*>(b), b_sk, b_sn, bias, bk, static_cast<float*>(d),
                   ldd, status, s);
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (a_sk != 1 && a_sm == 1 && m > 1) {
    // mat1 = X^T view of a row-major X [k, m] (the weight-gradient GEMM dW = dZ^T X): MN-major A
    if (epi != kEpiNone)
      return fail(GKO_ERR_UNSUPPORTED, "a transposed mat1 is supported without an activation only");
    if (b_sk == 1)
      return run_tc(dtype, epi, m, n, k, n, 0, a, a_sk, b, b_sn, false, bias, bk, d, ldd, status, s, nullptr,
                    nullptr, 0, nullptr, 0, nullptr, 0, nullptr, true);
    if (b_sn == 1)
      return run_tc(dtype, epi, m, n, k, n, 0, a, a_sk, b, b_sk, true, bias, bk, d, ldd, status, s, nullptr,
                    nullptr, 0, nullptr, 0, nullptr, 0, nullptr, true);
    return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs mat2 with unit stride in one dimension");
  }
  if (a_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED,
                "tensor-core GEMM needs mat1 with unit stride in one dimension (row-major, or a transposed "
                "view without an activation)");
  if (b_sk == 1) {
    // mat2 = W^T view of a row-major weight W [n, k]: K-major B.
    return run_tc(dtype, epi, m, n, k, n, 0, a, a_sm, b, b_sn, false, bias, bk, d, ldd, status, s);
  }
  if (b_sn == 1) {
    // mat2 stored row-major [k, n]: MN-major B.
    return run_tc(dtype, epi, m, n, k, n, 0, a, a_sm, b, b_sk, true, bias, bk, d, ldd, status, s);
  }
  return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs mat2 with unit stride in one dimension");
}

extern "C" int gko_linear_swiglu(int dtype, int64_t m, int64_t h, int64_t k, const void* x,
                                 int64_t x_sm, int64_t x_sk, const void* w, int64_t w_sn,
                                 int64_t w_sk, void* out, int64_t ldo, unsigned int* status,
                                 void* stream) {
  if (host::dtype_size(dtype) == 0) return fail(GKO_ERR_INVALID, "unknown dtype code %d", dtype);
  if (m < 0 || h < 0 || k < 0) return fail(GKO_ERR_INVALID, "negative GEMM size");
  if (m == 0 || h == 0) return GKO_OK;  // empty output: nothing is read or written
  if (!out || (k && (!x || !w))) return fail(GKO_ERR_INVALID, "null operand pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (m == 0 || h == 0) return GKO_OK;
  if (dtype == GKO_F32)
    // logical B[k, 2h] = W^T: strides (w_sk, w_sn)
    return run_f32(kEpiSwiglu, m, h, k, h, static_cast<const float*>(x), x_sm, x_sk,
                   static_cast<const float*>(w), w_sk, w_sn, nullptr, kBiasNone,
                   static_cast<float*>(out), ldo, status, s);
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (x_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED, "tensor-core SwiGLU needs a row-major x (stride(-1) == 1)");
  if (w_sk == 1)
    return run_tc(dtype, kEpiSwiglu, m, h, k, 2 * h, h, x, x_sm, w, w_sn, false, nullptr,
                  kBiasNone, out, ldo, status, s);
  if (w_sn == 1)
    return run_tc(dtype, kEpiSwiglu, m, h, k, 2 * h, h, x, x_sm, w, w_sk, true, nullptr,
                  kBiasNone, out, ldo, status, s);
  return fail(GKO_ERR_UNSUPPORTED, "tensor-core SwiGLU needs a weight with unit stride in one dim");
}

extern "C" int gko_linear_allreduce(int dtype, int64_t m, int64_t n, int64_t k, const void* x, int64_t x_sm,
                                    int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, void* out,
                                    int64_t ldo, void* out_multicast, void* const* out_peers, int world,
                                    unsigned int* status, void* stream) {
  if (dtype != GKO_BF16 && dtype != GKO_F16)
    return fail(GKO_ERR_UNSUPPORTED, "linear_allreduce takes bf16 or f16 (dtype code %d)", dtype);
  if (m < 0 || n < 0 || k < 0 || world < 1) return fail(GKO_ERR_INVALID, "negative size or world < 1");
  if (m == 0 || n == 0) return GKO_OK;
  if (!out || !x || !w) return fail(GKO_ERR_INVALID, "null operand pointer");
  if (!out_multicast && !out_peers)
    return fail(GKO_ERR_INVALID, "linear_allreduce needs a multicast address or the peers' output pointers");
  if (out_multicast && !host::aligned16(out_multicast))
    return fail(GKO_ERR_UNSUPPORTED, "linear_allreduce needs a 16-byte aligned multicast address");
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (x_sk != 1 || w_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED, "linear_allreduce needs row-major x [m, k] and weight [n, k]");
  return run_tc(dtype, kEpiAllReduce, m, n, k, n, 0, x, x_sm, w, w_sn, false, nullptr, kBiasNone, out, ldo, status,
                reinterpret_cast<cudaStream_t>(stream), out_multicast, out_peers, world);
}

extern "C" int gko_addmm_act_aux(int dtype, int act, int64_t m, int64_t n, int64_t k, const void* a, int64_t a_sm,
                                 int64_t a_sk, const void* b, int64_t b_sk, int64_t b_sn, const void* bias,
                                 int bias_dtype, void* d, int64_t ldd, void* z, int64_t ldz, unsigned int* status,
                                 void* stream) {
  if (dtype != GKO_BF16 && dtype != GKO_F16)
    return fail(GKO_ERR_UNSUPPORTED, "the pre-activation output is produced on the bf16 / f16 path only");
  if (act != GKO_ACT_NONE && act != GKO_ACT_GELU && act != GKO_ACT_RELU)
    return fail(GKO_ERR_INVALID, "unknown activation code %d", act);
  if (m < 0 || n < 0 || k < 0) return fail(GKO_ERR_INVALID, "negative GEMM size");
  if (m == 0 || n == 0) return GKO_OK;
  if (!d || !z || (k && (!a || !b))) return fail(GKO_ERR_INVALID, "null operand pointer");
  const int bk = bias_kind_of(bias, bias_dtype);
  if (bk < 0) return fail(GKO_ERR_INVALID, "unknown bias dtype code %d", bias_dtype);
  const int epi = act == GKO_ACT_GELU ? kEpiGelu : act == GKO_ACT_RELU ? kEpiRelu : kEpiNone;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (a_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs a row-major mat1 (stride(-1) == 1)");
  if (b_sk == 1)
    return run_tc(dtype, epi, m, n, k, n, 0, a, a_sm, b, b_sn, false, bias, bk, d, ldd, status, s, nullptr, nullptr,
                  0, z, ldz);
  if (b_sn == 1)
    return run_tc(dtype, epi, m, n, k, n, 0, a, a_sm, b, b_sk, true, bias, bk, d, ldd, status, s, nullptr, nullptr,
                  0, z, ldz);
  return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs mat2 with unit stride in one dimension");
}

extern "C" int gko_linear_swiglu_aux(int dtype, int64_t m, int64_t h, int64_t k, const void* x, int64_t x_sm,
                                     int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, void* out, int64_t ldo,
                                     void* gate_up, int64_t ldg, unsigned int* status, void* stream) {
  if (dtype != GKO_BF16 && dtype != GKO_F16)
    return fail(GKO_ERR_UNSUPPORTED, "the pre-activation output is produced on the bf16 / f16 path only");
  if (m < 0 || h < 0 || k < 0) return fail(GKO_ERR_INVALID, "negative GEMM size");
  if (m == 0 || h == 0) return GKO_OK;
  if (!out || !gate_up || (k && (!x || !w))) return fail(GKO_ERR_INVALID, "null operand pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (x_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED, "tensor-core SwiGLU needs a row-major x (stride(-1) == 1)");
  if (w_sk == 1)
    return run_tc(dtype, kEpiSwiglu, m, h, k, 2 * h, h, x, x_sm, w, w_sn, false, nullptr, kBiasNone, out, ldo, status,
                  s, nullptr, nullptr, 0, gate_up, ldg);
  if (w_sn == 1)
    return run_tc(dtype, kEpiSwiglu, m, h, k, 2 * h, h, x, x_sm, w, w_sk, true, nullptr, kBiasNone, out, ldo, status,
                  s, nullptr, nullptr, 0, gate_up, ldg);
  return fail(GKO_ERR_UNSUPPORTED, "tensor-core SwiGLU needs a weight with unit stride in one dim");
}

extern "C" int gko_linear_residual(int dtype, int64_t m, int64_t n, int64_t k, const void* x, int64_t x_sm,
                                   int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, const void* resid,
                                   int64_t resid_sm, void* out, int64_t ldo, unsigned int* status, void* stream) {
  if (dtype != GKO_BF16 && dtype != GKO_F16)
    return fail(GKO_ERR_UNSUPPORTED, "linear_residual runs on the bf16 / f16 tensor-core path only");
  if (m < 0 || n < 0 || k < 0) return fail(GKO_ERR_INVALID, "negative GEMM size");
  if (m == 0 || n == 0) return GKO_OK;
  if (!out || !resid || (k && (!x || !w))) return fail(GKO_ERR_INVALID, "null operand pointer");
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (x_sk != 1 || w_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED, "linear_residual needs row-major x [m, k] and weight [n, k]");
  return run_tc(dtype, kEpiNone, m, n, k, n, 0, x, x_sm, w, w_sn, false, nullptr, kBiasNone, out, ldo, status,
                reinterpret_cast<cudaStream_t>(stream), nullptr, nullptr, 0, nullptr, 0, resid, resid_sm);
}

extern "C" int gko_linear_rowscale(int dtype, int swiglu, int64_t m, int64_t n, int64_t k, const void* x,
                                   int64_t x_sm, int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk,
                                   const float* row_scale, void* out, int64_t ldo, unsigned int* status,
                                   void* stream) {
  if (dtype != GKO_BF16 && dtype != GKO_F16)
    return fail(GKO_ERR_UNSUPPORTED, "linear_rowscale runs on the bf16 / f16 tensor-core path only");
  if (m < 0 || n < 0 || k < 0) return fail(GKO_ERR_INVALID, "negative GEMM size");
  if (m == 0 || n == 0) return GKO_OK;
  if (!out || !row_scale || (k && (!x || !w))) return fail(GKO_ERR_INVALID, "null operand pointer");
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (x_sk != 1 || w_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED, "linear_rowscale needs row-major x [m, k] and weight [rows, k]");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (swiglu) {
    if (n % 8) return fail(GKO_ERR_UNSUPPORTED, "SwiGLU needs h %% 8 == 0");
    return run_tc(dtype, kEpiSwiglu, m, n, k, 2 * n, n, x, x_sm, w, w_sn, false, nullptr, kBiasNone, out, ldo,
                  status, s, nullptr, nullptr, 0, nullptr, 0, nullptr, 0, row_scale);
  }
  return run_tc(dtype, kEpiNone, m, n, k, n, 0, x, x_sm, w, w_sn, false, nullptr, kBiasNone, out, ldo, status, s,
                nullptr, nullptr, 0, nullptr, 0, nullptr, 0, row_scale);
}

extern "C" int gko_linear_rowscale_rope(int dtype, int64_t m, int64_t n, int64_t k, const void* x, int64_t x_sm,
                                        int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk,
                                        const float* row_scale, void* out, int64_t ldo, int64_t rope_cols,
                                        int64_t seq_len, float theta, unsigned int* status, void* stream) {
  if (dtype != GKO_BF16 && dtype != GKO_F16)
    return fail(GKO_ERR_UNSUPPORTED, "linear_rowscale_rope runs on the bf16 / f16 tensor-core path only");
  if (m < 0 || n < 0 || k < 0) return fail(GKO_ERR_INVALID, "negative GEMM size");
  if (rope_cols < 0 || rope_cols > n || rope_cols % 128 || seq_len <= 0 || seq_len >= (1ll << 31))
    return fail(GKO_ERR_INVALID, "rope_cols must be a multiple of 128 within n, and seq_len positive");
  if (!(theta > 1.f)) return fail(GKO_ERR_INVALID, "rope theta must be > 1");
  if (m == 0 || n == 0) return GKO_OK;
  if (!out || !row_scale || (k && (!x || !w))) return fail(GKO_ERR_INVALID, "null operand pointer");
  if (k == 0) return fail(GKO_ERR_UNSUPPORTED, "tensor-core GEMM needs k > 0");
  if (x_sk != 1 || w_sk != 1)
    return fail(GKO_ERR_UNSUPPORTED, "linear_rowscale_rope needs row-major x [m, k] and weight [rows, k]");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return run_tc(dtype, kEpiNone, m, n, k, n, 0, x, x_sm, w, w_sn, false, nullptr, kBiasNone, out, ldo, status, s,
                nullptr, nullptr, 0, nullptr, 0, nullptr, 0, row_scale, false, (int)rope_cols, (int)seq_len,
                log2f(theta));
}

extern "C" int gko_set_gemm_ctas(int ctas) {
  if (ctas < 0) {
    fail(GKO_ERR_INVALID, "gemm CTA limit must be >= 0 (0: every SM)");
    return -1;
  }
  return g_gemm_ctas.exchange(ctas);
}
