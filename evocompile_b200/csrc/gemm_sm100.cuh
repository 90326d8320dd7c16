// Persistent, warp-specialised tcgen05 GEMM with fused epilogues for sm_100a.
//
//   D[M, N_out] = epilogue( A[M, K] * B^T )      A: K-major (row-major [M, K])
//                                                 B: K-major ([N, K]) or MN-major ([K, N])
//
// Epilogues (the fused operators of the kernel catalog):
//   kEpiNone   : D = A*B^T (+ bias)                      down-projection / plain linear
//   kEpiGelu   : D = gelu_erf(A*B^T + bias)              gko::addmm_gelu
//   kEpiRelu   : D = relu(A*B^T + bias)
//   kEpiSwiglu : D = silu(A*Bg^T) * (A*Bu^T)             gko::gemm_swiglu, B = [Bg; Bu]
//   kEpiAllReduce: D_r += A*B^T on every rank r of a tensor-parallel group (row-parallel
//                linear + all-reduce in one kernel): each staged output chunk is added into
//                all ranks' D through the NVLink multicast address (in-switch reduction),
//                or through each peer's mapped D when no multicast object exists
//
// CTA = 10 warps: warp 0 TMA producer, warp 1 MMA issuer (+TMEM owner),
//                 warps 2..9 epilogue (TMEM -> registers -> smem -> TMA store); two
//                 warps per TMEM lane quarter, each converting half of the columns.
// Tile order: grouped raster chosen on the host so that the operand shared by a
// group of tiles stays resident in L2 (see GemmParams::group / raster_n).
// Tiles: 128 x 256 accumulator (SwiGLU: 128 gate + 128 up columns -> 128 outputs),
// K step 64 (one 128-byte swizzle row), 4-stage smem ring, two TMEM accumulators
// (2 x 256 columns) so the epilogue of tile i overlaps the main loop of tile i+1.
#pragma once

#include <type_traits>

#include "sm100_ptx.cuh"

namespace gko {

enum : int { kEpiNone = 0, kEpiGelu = 1, kEpiRelu = 2, kEpiSwiglu = 3, kEpiAllReduce = 4 };
enum : int { kBiasNone = 0, kBiasF16 = 1, kBiasBF16 = 2, kBiasF32 = 3 };

struct GemmParams {
  int M;            // rows of A / D
  int N_out;        // columns of D
  int K;            // reduction length
  int up_offset;    // SwiGLU: first row (K-major) / column (MN-major) of the up block in B
  int m_blocks;     // ceil(M / 128)
  int n_blocks;     // ceil(N_out / kBlockNOut)
  int num_tiles;    // m_blocks * n_blocks
  int k_blocks;     // ceil(K / 64)
  int group;        // raster: tiles sweep the other axis in groups of this many blocks
  int raster_n;     // 0: groups of M-blocks (A group stays in L2), 1: groups of N-blocks
  const void* bias;
  int bias_kind;
  unsigned* status;
  // kEpiAllReduce: destination D of every rank, by multicast address (red_mc) or, without
  // one, by the device array of the ranks' mapped D pointers (red_peers, red_world entries)
  void* red_mc;
  void* const* red_peers;
  int red_world;
  int64_t red_ld;  // row stride of D in elements
  // Optional second output for the backward (NULL: none): the pre-activation z = A*B^T + bias
  // (kEpiNone / kEpiGelu / kEpiRelu), or [gate | up] (kEpiSwiglu: gate in columns [0, N_out),
  // up in [N_out, 2 N_out)); row stride aux_ld elements.
  void* aux;
  int64_t aux_ld;
  // Optional residual R [M, N_out] (row stride resid_ld elements, NULL: none), added after the
  // activation: D = act(A*B^T + bias) + R (kEpiNone / kEpiGelu / kEpiRelu). D may be R.
  const void* resid;
  int64_t resid_ld;
  // Optional per-row scale s [M] (fp32, NULL: none) applied to the accumulator first:
  // D = act(s_r * (A*B^T) + bias) + R; SwiGLU: silu(s_r g) * (s_r u). With s = 1/rms(A row)
  // and the RMSNorm weight folded into B, the GEMM computes rmsnorm(A) * B^T.
  const float* row_scale;
  // Optional rotate-half RoPE (rope_cols > 0, kEpiNone, head dim 128): output columns
  // [0, rope_cols) are heads of 128 whose pairs (i, i + 64) are rotated by the angle
  // (row % rope_seq) * theta^(-2i/128) after the row scale, before rounding to T. The QKV
  // projection of a Llama block writes its q and k heads already rotated.
  int rope_cols;
  int rope_seq;
  float rope_log2_theta;
};

namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kMmaN = 256;
constexpr int kStages = 4;
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
constexpr uint32_t kABytes = kBM * kBK * 2;       // 16 KB
constexpr uint32_t kBBytes = kMmaN * kBK * 2;     // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kStagingBytes = kEpiWarps * 32 * 128;  // 8 warps x (32 rows x 128 B)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + kStagingBytes + 256;

__host__ __device__ constexpr int block_n_out(int epi) { return epi == kEpiSwiglu ? 128 : 256; }

// Grouped raster: consecutive tiles walk `group` blocks of one axis (fast) while
// sweeping the other, so concurrently running CTAs share operand tiles in L2.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& mb, int& nb) {
  const int fast_blocks = p.raster_n ? p.n_blocks : p.m_blocks;
  const int slow_blocks = p.raster_n ? p.m_blocks : p.n_blocks;
  const int group_size = p.group * slow_blocks;
  const int g = tile / group_size;
  const int first = g * p.group;
  const int gsz = min(p.group, fast_blocks - first);
  const int r = tile - g * group_size;
  const int fast = first + r % gsz;
  const int slow = r / gsz;
  mb = p.raster_n ? slow : fast;
  nb = p.raster_n ? fast : slow;
}

__device__ __forceinline__ float load_bias(const void* bias, int kind, int col, int n) {
  if (kind == kBiasNone || col >= n) return 0.f;
  if (kind == kBiasF32) return __ldg(reinterpret_cast<const float*>(bias) + col);
  if (kind == kBiasBF16)
    return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(bias) + col));
  return __half2float(__ldg(reinterpret_cast<const __half*>(bias) + col));
}

// Exact-erf GELU with CUDA's erff (the fp32 path, whose contract is rel 1e-3 with TF32 off).
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
}

// Exact-erf GELU for the bf16 / f16 epilogue, on a packed pair, with erf evaluated by
// Abramowitz & Stegun 7.1.28 (Handbook of Mathematical Functions, 1964):
//   erf(z) = 1 - 1 / (1 + a1 z + a2 z^2 + ... + a6 z^6)^16   for z >= 0 (odd extension below),
// maximum absolute error 3e-7, far below the bf16 rounding of the output (2^-9 relative). The
// polynomial and the 16th power run as f32x2 FMAs / multiplies, the reciprocal on the MUFU (one
// per element; for large z the power overflows to +inf and the reciprocal gives 0). The
// epilogue's issue slots are shared with the MMA-issuing warp, and on B200 CUDA's erff made the
// GELU epilogue cost 4-8 % of the GEMM's time at K = 4096 and 15 % at K = 1024.
__device__ __forceinline__ uint64_t gelu_erf_pair(uint64_t x) {
  constexpr float kInvSqrt2 = 0.70710678118654752f;
  float x0, x1;
  f2unpack(x, x0, x1);
  const uint64_t z = f2pack(fabsf(x0) * kInvSqrt2, fabsf(x1) * kInvSqrt2);
  uint64_t q = fma2(z, f2pack(0.0000430638f, 0.0000430638f), f2pack(0.0002765672f, 0.0002765672f));
  q = fma2(q, z, f2pack(0.0001520143f, 0.0001520143f));
  q = fma2(q, z, f2pack(0.0092705272f, 0.0092705272f));
  q = fma2(q, z, f2pack(0.0422820123f, 0.0422820123f));
  q = fma2(q, z, f2pack(0.0705230784f, 0.0705230784f));
  q = fma2(q, z, f2pack(1.f, 1.f));
  q = mul2(q, q);  // ^2
  q = mul2(q, q);  // ^4
  q = mul2(q, q);  // ^8
  q = mul2(q, q);  // ^16
  float q0, q1, r0, r1;
  f2unpack(q, q0, q1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(q0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(q1));
  // 0.5 x (1 + sign(x) (1 - r))
  const float e0 = copysignf(1.f - r0, x0), e1 = copysignf(1.f - r1, x1);
  return mul2(f2pack(0.5f * x0, 0.5f * x1), f2pack(1.f + e0, 1.f + e1));
}

// 32 bias values for columns [col, col + 32) (zeros past n), the same for every lane: uniform
// 16-byte loads that the L1 broadcasts, in place of one shuffle per output element.
__device__ __forceinline__ void load_bias32(const void* bias, int kind, int col, int n, float (&b)[32]) {
  if (kind == kBiasF32) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col + 4 * j < n) v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(bias) + col) + j);
      b[4 * j] = v.x;
      b[4 * j + 1] = v.y;
      b[4 * j + 2] = v.z;
      b[4 * j + 3] = v.w;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (col + 8 * j < n)
      v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(bias) + col) + j);
    auto put = [&](uint32_t word, int e) {
      float lo, hi;
      if (kind == kBiasBF16)
        Cvt<__nv_bfloat16>::unpack(word, lo, hi);
      else
        Cvt<__half>::unpack(word, lo, hi);
      b[8 * j + 2 * e] = lo;
      b[8 * j + 2 * e + 1] = hi;
    };
    put(v.x, 0);
    put(v.y, 1);
    put(v.z, 2);
    put(v.w, 3);
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// Converts this warp's half of one accumulator tile (32 TMEM lanes starting at
// t_row) into the output: TMEM -> registers -> epilogue math -> 128B-swizzled
// staging buffer -> TMA store of [32 rows x 64 columns] per chunk. With p.aux set, the
// pre-activation of the same chunk (for SwiGLU its gate and its up columns) is then read again
// from TMEM, staged through the same buffer and TMA-stored through tm_x0 (gate / the only
// pre-activation) and tm_x1 (up). Calls `release()` (on one lane, after the warp's last TMEM
// read of the tile) so the MMA warp may reuse the accumulator.

// Reads 32 values of row `row` from column `col` (16-byte loads; zeros past M / N).
template <typename T>
__device__ __forceinline__ void load_row32(const void* src, int64_t ld, int row, int col, int M, int N,
                                           uint32_t (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = 0u;
  if (row >= M) return;
  const T* s = static_cast<const T*>(src) + (int64_t)row * ld + col;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (col + 8 * j < N) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(s) + j);
      v[4 * j] = q.x;
      v[4 * j + 1] = q.y;
      v[4 * j + 2] = q.z;
      v[4 * j + 3] = q.w;
    }
}

// Writes 32 packed values (this lane's row, columns [h * 32, h * 32 + 32) of the chunk) into
// the 128B-swizzled staging row: 16-byte piece j of row `lane` lives at j ^ (lane & 7).
__device__ __forceinline__ void stage_row32(uint32_t buf, int lane, int h, const uint32_t (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int piece = h * 4 + j;
    const uint32_t addr = buf + lane * 128 + ((piece ^ (lane & 7)) << 4);
    st_shared_v4(addr, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

// TMA store of the staged [32 rows x 64 columns] to (col, row0) through `tm` (lane 0).
__device__ __forceinline__ void store_staged(const CUtensorMap* tm, uint32_t buf, int col, int row0, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d_hint(tm, buf, col, row0, l2_policy_evict_first());
    bulk_commit_group();
  }
}

template <typename T, int EPI, typename Release>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const CUtensorMap* tm_d,
                                              const CUtensorMap* tm_x0, const CUtensorMap* tm_x1,
                                              uint32_t t_row, int row0, int col_base, int half,
                                              uint32_t buf, int lane, Release release) {
  constexpr int kBNOut = block_n_out(EPI);
  constexpr int kChunks = kBNOut / 64;
  constexpr int kMyChunks = kChunks / 2;
#pragma unroll 1
  for (int cc = 0; cc < kMyChunks; ++cc) {
    const int c = half * kMyChunks + cc;
    // the previous store from this warp's staging buffer must have read it
    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col0 = c * 64 + h * 32;
      uint32_t packed[16];
      const float rs = (p.row_scale && row0 + lane < p.M) ? __ldg(p.row_scale + row0 + lane) : 1.f;
      if constexpr (EPI == kEpiSwiglu) {
        uint32_t g[32], u[32];
        tmem_ld32(t_row + col0, g);
        tmem_ld32(t_row + 128 + col0, u);
        tmem_wait_ld();
        if (p.row_scale) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            g[i] = __float_as_uint(__uint_as_float(g[i]) * rs);
            u[i] = __float_as_uint(__uint_as_float(u[i]) * rs);
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float g0 = __uint_as_float(g[2 * i]), g1 = __uint_as_float(g[2 * i + 1]);
          const float u0 = __uint_as_float(u[2 * i]), u1 = __uint_as_float(u[2 * i + 1]);
          packed[i] = Cvt<T>::pack(silu(g0) * u0, silu(g1) * u1);
        }
      } else if (EPI == kEpiNone && p.rope_cols > 0 && col_base + c * 64 < p.rope_cols) {
        // this chunk is one half of a 128-column head: its partner half is 64 columns away
        const int hi = cc;  // 0: columns i of the head, 1: columns i + 64
        uint32_t v[32], w[32];
        tmem_ld32(t_row + col0, v);
        tmem_ld32(t_row + col0 + (hi ? -64 : 64), w);
        tmem_wait_ld();
        const float pos = (float)((row0 + lane) % p.rope_seq);
        const int i0 = (col0 & 63);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float o[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int idx = i0 + 2 * i + e;
            const float inv_freq = exp2f(-p.rope_log2_theta * (2.f * (float)idx / 128.f));
            float sn, cs;
            sincosf(pos * inv_freq, &sn, &cs);
            const float x = __uint_as_float(v[2 * i + e]) * rs, y = __uint_as_float(w[2 * i + e]) * rs;
            o[e] = hi ? fmaf(x, cs, y * sn) : fmaf(x, cs, -y * sn);
          }
          packed[i] = Cvt<T>::pack(o[0], o[1]);
        }
      } else {
        uint32_t v[32];
        tmem_ld32(t_row + col0, v);
        // the bias of these 32 columns (read while the TMEM load is in flight)
        float bv[32];
        if (p.bias_kind != kBiasNone) {
          load_bias32(p.bias, p.bias_kind, col_base + col0, p.N_out, bv);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) bv[i] = 0.f;
        }
        uint32_t rv[16];  // this lane's row of the residual
        if (p.resid) load_row32<T>(p.resid, p.resid_ld, row0 + lane, col_base + col0, p.M, p.N_out, rv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0 = fmaf(__uint_as_float(v[2 * i]), rs, bv[2 * i]);
          float x1 = fmaf(__uint_as_float(v[2 * i + 1]), rs, bv[2 * i + 1]);
          if constexpr (EPI == kEpiGelu) {
            f2unpack(gelu_erf_pair(f2pack(x0, x1)), x0, x1);
          } else if constexpr (EPI == kEpiRelu) {
            x0 = fmaxf(x0, 0.f);
            x1 = fmaxf(x1, 0.f);
          }
          if (p.resid) {
            float r0, r1;
            Cvt<T>::unpack(rv[i], r0, r1);
            x0 += r0;
            x1 += r1;
          }
          packed[i] = Cvt<T>::pack(x0, x1);
        }
      }
      stage_row32(buf, lane, h, packed);
    }
    // with a pre-activation output the accumulator is read again below, so it is released
    // after those reads
    if (cc == kMyChunks - 1 && !p.aux) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) release();
    }
    if constexpr (EPI == kEpiAllReduce) {
      // row-contiguous read-back of the staged [32 rows x 64 columns]: 8 lanes per row, so a
      // warp instruction adds four 128-byte row segments
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + (lane >> 3), j = lane & 7;
        const uint4 v = ld_shared_v4(buf + r * 128 + ((j ^ (r & 7)) << 4));
        const int grow = row0 + r, gcol = col_base + c * 64 + j * 8;
        if (grow < p.M && gcol < p.N_out) {
          const int64_t off = ((int64_t)grow * p.red_ld + gcol) * (int64_t)sizeof(T);
          if (p.red_mc) {
            multimem_red_add_x8<T>(static_cast<uint8_t*>(p.red_mc) + off, v);
          } else {
            for (int w = 0; w < p.red_world; ++w) red_add_x8<T>(static_cast<uint8_t*>(p.red_peers[w]) + off, v);
          }
        }
      }
      __syncwarp();
    } else {
      store_staged(tm_d, buf, col_base + c * 64, row0, lane);
      if (p.aux) {
        // the pre-activation of this chunk, one staged [32 x 64] box per part (SwiGLU: gate, up)
        constexpr int kParts = EPI == kEpiSwiglu ? 2 : 1;
#pragma unroll 1
        for (int part = 0; part < kParts; ++part) {
          if (lane == 0) bulk_wait_group_read<0>();  // the previous store has read the buffer
          __syncwarp();
          const float rs = (p.row_scale && row0 + lane < p.M) ? __ldg(p.row_scale + row0 + lane) : 1.f;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int col0 = c * 64 + h * 32;
            uint32_t v[32];
            tmem_ld32(t_row + part * 128 + col0, v);
            float bv[32];
            if (EPI != kEpiSwiglu && p.bias_kind != kBiasNone) {
              load_bias32(p.bias, p.bias_kind, col_base + col0, p.N_out, bv);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) bv[i] = 0.f;
            }
            tmem_wait_ld();
            uint32_t z[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              z[i] = Cvt<T>::pack(fmaf(__uint_as_float(v[2 * i]), rs, bv[2 * i]),
                                  fmaf(__uint_as_float(v[2 * i + 1]), rs, bv[2 * i + 1]));
            stage_row32(buf, lane, h, z);
          }
          store_staged(part ? tm_x1 : tm_x0, buf, col_base + c * 64, row0, lane);
        }
        if (cc == kMyChunks - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release();
        }
      }
    }
  }
}

// A_MN: A stored MN-major ([K, M] row-major, e.g. the transposed view of an activation
// gradient dZ [tokens, N] when the GEMM computes dW = dZ^T X over the token axis): each stage
// holds two 64-row M chunks of 64 K-rows, like the MN-major B tile.
template <typename T, int EPI, bool B_MN, bool A_MN = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_d, const __grid_constant__ CUtensorMap tm_x0,
                const __grid_constant__ CUtensorMap tm_x1, const GemmParams p) {
  constexpr int kBNOut = block_n_out(EPI);
  constexpr uint32_t kIdesc =
      make_idesc_f16(std::is_same<T, __nv_bfloat16>::value, kBM, kMmaN, A_MN, B_MN);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_addr + pad;
  const uint32_t sA = sbase;
  const uint32_t sB = sA + kStages * kABytes;
  const uint32_t sStage = sB + kStages * kBBytes;
  uint8_t* meta = smem + kStages * kStageBytes + kStagingBytes;
  const uint32_t smeta = sStage + kStagingBytes;
  // barriers: full[4] empty[4] tfull[2] tempty[2] drain
  const uint32_t bar_full = smeta;
  const uint32_t bar_empty = smeta + 8 * kStages;
  const uint32_t bar_tfull = smeta + 16 * kStages;
  const uint32_t bar_tempty = bar_tfull + 16;
  const uint32_t bar_drain = bar_tempty + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(meta + 16 * kStages + 40);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 16 * kStages + 48);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, kEpiWarps);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_d);
    if (p.aux) {
      prefetch_tmap(&tm_x0);
      if (EPI == kEpiSwiglu) prefetch_tmap(&tm_x1);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // the operand a raster group shares stays in L2; the streamed one goes first
      const uint64_t keep = l2_policy_evict_last(), stream = l2_policy_evict_first();
      const uint64_t pol_a = p.raster_n ? stream : keep, pol_b = p.raster_n ? keep : stream;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(p, tile, mb, nb);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag, p.status,
                            kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t full = bar_full + 8 * stage;
          mbar_arrive_expect_tx(full, kStageBytes);
          const uint32_t a_dst = sA + stage * kABytes;
          const uint32_t b_dst = sB + stage * kBBytes;
          const int k0 = kb * kBK;
          if constexpr (A_MN) {
            // A is [K, M] MN-major: two 64-column boxes, 64 K-rows each.
            tma_load_2d_hint(a_dst, &tm_a, full, mb * kBM, k0, pol_a);
            tma_load_2d_hint(a_dst + kABytes / 2, &tm_a, full, mb * kBM + 64, k0, pol_a);
          } else {
            tma_load_2d_hint(a_dst, &tm_a, full, k0, mb * kBM, pol_a);
          }
          if constexpr (!B_MN) {
            // B is [N, K] K-major: two 128-row boxes.
            if constexpr (EPI == kEpiSwiglu) {
              tma_load_2d_hint(b_dst, &tm_b, full, k0, nb * 128, pol_b);
              tma_load_2d_hint(b_dst + kBBytes / 2, &tm_b, full, k0, p.up_offset + nb * 128, pol_b);
            } else {
              tma_load_2d_hint(b_dst, &tm_b, full, k0, nb * 256, pol_b);
              tma_load_2d_hint(b_dst + kBBytes / 2, &tm_b, full, k0, nb * 256 + 128, pol_b);
            }
          } else {
            // B is [K, N] MN-major: four 64-column boxes, 64 K-rows each.
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              int col;
              if constexpr (EPI == kEpiSwiglu)
                col = (c < 2) ? nb * 128 + c * 64 : p.up_offset + nb * 128 + (c - 2) * 64;
              else
                col = nb * 256 + c * 64;
              tma_load_2d_hint(b_dst + c * (kBBytes / 4), &tm_b, full, col, k0, pol_b);
            }
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      // Descriptors are built once: a stage or a K step only adds a constant to the 14-bit
      // start-address field (shared-memory addresses stay below 256 KB, so it never carries);
      // building them per MMA costs the issuing thread more than an MMA's execution time.
      const uint64_t d_a0 = A_MN ? make_sdesc_sw128(sA, kABytes / 2, 1024) : make_sdesc_sw128(sA, 16, 1024);
      const uint64_t d_b0 = B_MN ? make_sdesc_sw128(sB, kBBytes / 4, 1024) : make_sdesc_sw128(sB, 16, 1024);
      constexpr uint32_t kKStepA = A_MN ? (16 * 128) >> 4 : 32 >> 4;  // per K16 step, 16-byte units
      constexpr uint32_t kKStepB = B_MN ? (16 * 128) >> 4 : 32 >> 4;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_bounded(bar_tempty + 8 * acc, acc_phase ^ 1, abort_flag, p.status,
                          kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kMmaN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bounded(bar_full + 8 * stage, phase, abort_flag, p.status,
                            kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_st = d_a0 + (uint64_t)(stage * (kABytes >> 4));
          const uint64_t b_st = d_b0 + (uint64_t)(stage * (kBBytes >> 4));
          const uint32_t acc0 = kb != 0 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_f16_ss(d_tmem, a_st + kk * kKStepA, b_st + kk * kKStepB, kIdesc, kk > 0 ? 1u : acc0);
          mma_commit(bar_empty + 8 * stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(bar_tfull + 8 * acc);
      }
      if (*abort_flag) {
        // Drain this thread's tensor-core work before the TMEM is released.
        mma_commit(bar_drain);
        wait_for(bar_drain, 0, p.status, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;        // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;    // which half of the tile's columns it converts
    const uint32_t buf = sStage + (warp - 2) * (32 * 128);
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(p, tile, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!wait_bounded(bar_tfull + 8 * acc, acc_phase, abort_flag, p.status,
                        kStatusTimeoutEpilogue))
        break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * kMmaN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int row0 = mb * kBM + quarter * 32;
      const int col_base = nb * kBNOut;
      epilogue_tile<T, EPI>(p, &tm_d, &tm_x0, &tm_x1, t_row, row0, col_base, half, buf, lane,
                            [&] { mbar_arrive(bar_tempty + 8 * acc); });
    }
    if (lane == 0) bulk_wait_group<0>();
    // cross-GPU reductions are performed at system scope before the kernel is seen as done
    if constexpr (EPI == kEpiAllReduce) __threadfence_system();
    __syncwarp();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}


// ---------------------------------------------------------------------------
// CTA-pair version (cta_group::2): a cluster of two CTAs on neighbouring SMs
// computes a 256 x 256 accumulator tile. CTA r of the pair loads rows
// [128 r, 128 r + 128) of the A tile and columns [128 r, 128 r + 128) of the
// B tile (SwiGLU: CTA 0 the gate columns, CTA 1 the up columns) into its own
// shared memory; the leader (r = 0) issues M = 256 MMAs that read both CTAs'
// operands and write each CTA's 128 accumulator rows into that CTA's TMEM. Each
// SM therefore streams half of B per MMA: 64 instead of 96 bytes of shared
// memory per tensor-core cycle, and a third less L2 traffic.
//   full[s]   (leader only)  both CTAs' TMA bytes for stage s; leader's producer arrives
//   empty[s]  (both)         leader's MMA commit to each CTA when stage s is consumed
//   tfull[a]  (both)         leader's MMA commit to each CTA when accumulator a is done
//   tempty[a] (leader only)  16 epilogue warps (8 per CTA) release accumulator a
// No TMA multicast: every CTA loads its own operands.
constexpr int kPairStages = 6;
constexpr uint32_t kPairStageBytes = 2 * 128 * kBK * 2;  // A half + B half: 32 KB
constexpr uint32_t kPairSmemBytes = 1024 + kPairStages * kPairStageBytes + kStagingBytes + 256;

template <typename T, int EPI, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_d, const GemmParams p) {
  constexpr int kBNOut = block_n_out(EPI);
  constexpr uint32_t kIdesc =
      make_idesc_f16(std::is_same<T, __nv_bfloat16>::value, 2 * kBM, kMmaN, false, B_MN);
  constexpr uint32_t kHalfBytes = 128 * kBK * 2;  // 16 KB
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sbase = raw_addr + pad;
  const uint32_t sA = sbase;                               // [stages][128 x 64]
  const uint32_t sB = sA + kPairStages * kHalfBytes;      // [stages][128 x 64]
  const uint32_t sStage = sB + kPairStages * kHalfBytes;
  uint8_t* meta = smem + kPairStages * kPairStageBytes + kStagingBytes;
  const uint32_t smeta = sStage + kStagingBytes;
  const uint32_t bar_full = smeta;                      // [6]
  const uint32_t bar_empty = smeta + 8 * kPairStages;   // [6]
  const uint32_t bar_tfull = smeta + 16 * kPairStages;  // [2]
  const uint32_t bar_tempty = bar_tfull + 16;           // [2]
  const uint32_t bar_drain = bar_tempty + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(meta + 16 * kPairStages + 40);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 16 * kPairStages + 48);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int st = 0; st < kPairStages; ++st) {
      mbar_init(bar_full + 8 * st, 1);
      mbar_init(bar_empty + 8 * st, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, 2 * kEpiWarps);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_d);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t keep = l2_policy_evict_last(), stream = l2_policy_evict_first();
      const uint64_t pol_a = p.raster_n ? stream : keep, pol_b = p.raster_n ? keep : stream;
      for (int tile = cluster; tile < p.num_tiles && ok; tile += clusters) {
        int mb, nb;
        tile_coords(p, tile, mb, nb);
        const int row_a = mb * 2 * kBM + (int)rank * kBM;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bounded_cluster(bar_empty + 8 * stage, phase ^ 1, abort_flag, p.status,
                                    kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t full_local = bar_full + 8 * stage;
          const uint32_t full_leader = mapa_shared(full_local, 0);
          if (leader) mbar_arrive_expect_tx(full_local, 2 * kPairStageBytes);
          const int k0 = kb * kBK;
          tma_load_2d_pair_hint(sA + stage * kHalfBytes, &tm_a, full_leader, k0, row_a, pol_a);
          const uint32_t b_dst = sB + stage * kHalfBytes;
          if constexpr (!B_MN) {
            int brow;
            if constexpr (EPI == kEpiSwiglu)
              brow = rank ? p.up_offset + nb * 128 : nb * 128;
            else
              brow = nb * 256 + (int)rank * 128;
            tma_load_2d_pair_hint(b_dst, &tm_b, full_leader, k0, brow, pol_b);
          } else {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              int col;
              if constexpr (EPI == kEpiSwiglu)
                col = (rank ? p.up_offset : 0) + nb * 128 + c * 64;
              else
                col = nb * 256 + (int)rank * 128 + c * 64;
              tma_load_2d_pair_hint(b_dst + c * (kHalfBytes / 2), &tm_b, full_leader, col, k0, pol_b);
            }
          }
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = cluster; tile < p.num_tiles && ok; tile += clusters, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_bounded_cluster(bar_tempty + 8 * acc, acc_phase ^ 1, abort_flag, p.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kMmaN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bounded(bar_full + 8 * stage, phase, abort_flag, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sA + stage * kHalfBytes;
          const uint32_t b_addr = sB + stage * kHalfBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = make_sdesc_sw128(a_addr + kk * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (!B_MN)
              bdesc = make_sdesc_sw128(b_addr + kk * 32, 16, 1024);
            else
              bdesc = make_sdesc_sw128(b_addr + kk * 16 * 128, kHalfBytes / 2, 1024);
            mma_f16_ss_pair(d_tmem, adesc, bdesc, kIdesc, (kb | kk) != 0);
          }
          // release stage `stage` in both CTAs once these MMAs have read it
          mma_commit_pair(bar_empty + 8 * stage);
          mma_commit_pair(mapa_shared(bar_empty + 8 * stage, 1));
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(bar_tfull + 8 * acc);
        mma_commit_pair(mapa_shared(bar_tfull + 8 * acc, 1));
      }
      if (*abort_flag) {
        mma_commit_pair(bar_drain);
        wait_for(bar_drain, 0, p.status, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t buf = sStage + (warp - 2) * (32 * 128);
    int local = 0;
    for (int tile = cluster; tile < p.num_tiles; tile += clusters, ++local) {
      int mb, nb;
      tile_coords(p, tile, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!wait_bounded_cluster(bar_tfull + 8 * acc, acc_phase, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * kMmaN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int row0 = mb * 2 * kBM + (int)rank * kBM + quarter * 32;
      const uint32_t tempty_leader = mapa_shared(bar_tempty + 8 * acc, 0);
      // the pair path never writes a pre-activation (the host keeps aux launches single-CTA)
      epilogue_tile<T, EPI>(p, &tm_d, &tm_d, &tm_d, t_row, row0, nb * kBNOut, half, buf, lane,
                            [&] { mbar_arrive_cluster(tempty_leader); });
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // all MMAs done and all cross-CTA signals delivered before teardown
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

}  // namespace gemm
}  // namespace gko
