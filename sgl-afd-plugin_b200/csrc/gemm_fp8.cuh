// FP8 E4M3 experts with fp32 scales per 128 x 128 weight block (SGLang's block-quantised FusedMoE format,
// python/sgl_asap_plugin/srt/managers/scheduler.py:410-412 -> FusedMoE with a DeepSeek-style FP8 checkpoint):
// per-token 1 x 128 activation quantisation, the expert-major copy, and the two grouped GEMMs on tcgen05
// kind::f8f6f4.  Included by ffn.cu (same translation unit: JobDesc, QuantArgs, gemm::decode_tile).
//
// Block scales are not powers of two, so they cannot ride in the MMA: every 128-deep K block is accumulated
// on its own into one of two TMEM buffers (ping-pong), and the epilogue warps fold it into fp32 registers,
//     acc[r][c] += partial_kb[r][c] * (sa[r][kb] * sb[c / 128][kb]),
// while the tensor core already runs the next K block into the other buffer.

namespace gemm8 {
constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;  // E4M3 activations, 128 rows x 128 bytes
constexpr int B_BYTES = BN * BK;  // E4M3 weights, 256 rows x 128 bytes (two 128-row boxes)
constexpr int B_HALF = B_BYTES / 2;
constexpr uint32_t STAGE_TX = A_BYTES + B_BYTES;
constexpr int NUM_EPI_WARPS = 8;
// GEMM1 runs 12 warps: warpgroup 0 (TMA producer, MMA issuer, two idle warps) gives registers up with setmaxnreg
// (48 each) so the two epilogue warpgroups can hold 224 (the fp32 promotion accumulators plus two TMEM loads in
// flight): 128 x 48 + 256 x 224 = 63488 <= 384 x 168 registers at launch.  GEMM2 keeps 10 warps (no split: it
// measured slower with it).
template <int EPI>
struct Cfg {
  static constexpr int EPI_BASE = EPI == 0 ? 4 : 2;  // first epilogue warp
  static constexpr int THREADS = 32 * (EPI_BASE + NUM_EPI_WARPS);
};
constexpr uint32_t TMEM_COLS = 512;  // two 256-column partial accumulators
constexpr int CTRL_BYTES = 4096;     // barriers, TMEM slot, expert starts, row amax exchange
constexpr int STAGE_OUT_BYTES = NUM_EPI_WARPS * 2048;  // GEMM2 output staging, 32 rows x 64 B per epilogue warp
constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES) + STAGE_OUT_BYTES + CTRL_BYTES;
static_assert(SMEM_BYTES <= 232448, "shared memory over the 227 KB per block");
static_assert(256 + 4 * (ASAP_MAX_LOCAL_EXPERTS + 1) <= 1536, "expert starts overlap the tile queue");
constexpr int TILE_Q = 8;  // dynamic tile scheduler queue (as gemm::moe_gemm_kernel), at ctrl + 1536
constexpr float kE4M3Max = 448.f;

// tcgen05 instruction descriptor, kind::f8f6f4: D fp32, A = B = E4M3, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f8f6f4(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct Params {
  CUtensorMap tmap_a;  // activations [m_cap, K] E4M3
  CUtensorMap tmap_b;  // weights [P * N, K] E4M3, the checkpoint's row order
  const float* sa;     // activation scales, K-block-major [K/128][m_cap]
  const float* sb;     // weight block scales [P][N/128][K/128]
  int64_t m_cap;
  const JobDesc* desc;
  const int32_t* mstart;   // [P + 1] in 128-row blocks
  const int32_t* row_tok;  // [m_cap]
  const float* row_w;      // [m_cap]
  uint8_t* out_q;          // GEMM1: [m_cap, N/2] E4M3
  float* out_sa;           // GEMM1: [(N/2)/128][m_cap] fp32
  __nv_bfloat16* out_bf;   // GEMM2: [m_cap, N]
  uint32_t* tile_ctr;      // the job's tile counter of this GEMM (JobDesc::tiles)
  int32_t P, N, K;
  float swiglu_limit;
  uint64_t status, timeout_ns;
};

// acc[i] += x[i] * f for 32 consecutive accumulators, two per instruction (the packed fp32 FMA of sm_100; each
// lane is one fused multiply-add with one rounding, the same result as fmaf): the promotion of a K block is
// FMA-issue-bound next to the TMEM loads, and the pairs halve its issue slots.
__device__ __forceinline__ void fma32_pairs(float* acc, const uint32_t (&x)[32], float f) {
  const float2 ff = make_float2(f, f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 r = __ffma2_rn(make_float2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])), ff,
                                make_float2(acc[2 * i], acc[2 * i + 1]));
    acc[2 * i] = r.x;
    acc[2 * i + 1] = r.y;
  }
}

// E4M3 codes of 4 values (scaled by inv) packed little-endian into one word.
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d, float inv) {
  return cvt_e4m3x2(a * inv, b * inv) | (cvt_e4m3x2(c * inv, d * inv) << 16);
}

// EPI 0 (GEMM1, N = 2I): tile n covers gate rows [128n, 128n+128) and up rows I + [128n, 128n+128); epilogue
// h = silu(gate) * up, requantised to E4M3 per 1 x 128 (the tile's 128 h columns are one K block of GEMM2).
// EPI 1 (GEMM2, N = H): tile n covers rows [256n, 256n+256); epilogue bf16(acc * w[row]).
template <int EPI>
__global__ void __launch_bounds__(Cfg<EPI>::THREADS, 1) moe_gemm_fp8_kernel(const __grid_constant__ Params p) {
  constexpr int THREADS = Cfg<EPI>::THREADS, EPI_BASE = Cfg<EPI>::EPI_BASE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * B_BYTES;
  uint8_t* ctrl = sOut + STAGE_OUT_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint64_t* amax_bar = mma_done + 1;    // [4 lane quarters][2 tile parities]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + 192);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctrl + 196);
  int32_t* s_mstart = reinterpret_cast<int32_t*>(ctrl + 256);
  uint64_t* tq_full = reinterpret_cast<uint64_t*>(ctrl + 1536);  // [TILE_Q] a tile index was published
  uint64_t* tq_empty = tq_full + TILE_Q;                          // [TILE_Q] every consumer warp has read it
  int32_t* s_tile = reinterpret_cast<int32_t*>(tq_empty + TILE_Q);
  float* s_amax = reinterpret_cast<float*>(ctrl + 2048);  // [2 tile parities][2 halves][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = p.P;
  const bool valid_job = p.desc->valid != 0;
  for (int i = threadIdx.x; i <= P; i += THREADS) s_mstart[i] = valid_job ? p.mstart[i] : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], NUM_EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    for (int b = 0; b < 8; ++b) mbar_init(&amax_bar[b], 64);
    for (int q = 0; q < TILE_Q; ++q) {
      mbar_init(&tq_full[q], 1);
      mbar_init(&tq_empty[q], 1 + NUM_EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmap_a);
    prefetch_tmap(&p.tmap_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int NT = p.N / BN, KT = p.K / BK;
  const int num_tiles = s_mstart[P] * NT;
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

  if (warp < EPI_BASE) {
  if constexpr (EPI == 0) asm volatile("setmaxnreg.dec.sync.aligned.u32 48;\n" ::: "memory");
  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (uint32_t tq = 0; ok; ++tq) {
        // claim the next tile and publish it (-1: none left) to the MMA and epilogue warps
        const int q = tq % TILE_Q;
        if (!mbar_wait(&tq_empty[q], ((tq / TILE_Q) & 1u) ^ 1u, deadline, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t claimed = atomicAdd(p.tile_ctr, 1u);
        const int tile = claimed < (uint32_t)num_tiles ? (int)claimed : -1;
        s_tile[q] = tile;
        mbar_arrive(&tq_full[q]);
        if (tile < 0) break;
        int e, m_blk, n_t;
        gemm::decode_tile(s_mstart, P, NT, tile, e, m_blk, n_t);
        const int a_row = m_blk * BM;
        int b0, b1;
        if constexpr (EPI == 0) {
          b0 = e * p.N + n_t * 128;
          b1 = e * p.N + p.N / 2 + n_t * 128;
        } else {
          b0 = e * p.N + n_t * BN;
          b1 = b0 + 128;
        }
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, deadline, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_TX);
          tma_load_2d(sA + stage * A_BYTES, &p.tmap_a, kt * BK, a_row, &full[stage]);
          tma_load_2d(sB + stage * B_BYTES, &p.tmap_b, kt * BK, b0, &full[stage]);
          tma_load_2d(sB + stage * B_BYTES + B_HALF, &p.tmap_b, kt * BK, b1, &full[stage]);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: the copies of the last armed stages must land before this CTA may exit.
      const uint64_t drain_deadline = globaltimer_ns() + 200000000ull;
      const int n_drain = issued < STAGES ? issued : STAGES;
      volatile int no_abort = 0;
      for (int i = 0; i < n_drain; ++i) {
        int s = stage - 1 - i;
        uint32_t ph = phase;
        if (s < 0) {
          s += STAGES;
          ph ^= 1u;
        }
        mbar_wait(&full[s], ph, drain_deadline, &no_abort);
      }
      if (!ok) report(p.status, status_word(ASAP_ST_PIPELINE_TIMEOUT, 0, 0, 8 + EPI));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one K block per TMEM buffer, alternating
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t it = 0;
      const uint32_t idesc = idesc_f8f6f4(BM, BN);
      bool ok = true;
      for (uint32_t tq = 0; ok; ++tq) {
        const int q = tq % TILE_Q;
        if (!mbar_wait(&tq_full[q], (tq / TILE_Q) & 1u, deadline, abort_flag)) break;
        const int tile = s_tile[q];
        mbar_arrive(&tq_empty[q]);
        if (tile < 0) break;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const uint32_t buf = it & 1u;
          if (!mbar_wait(&acc_empty[buf], ((it >> 1) & 1u) ^ 1u, deadline, abort_flag) ||
              !mbar_wait(&full[stage], phase, deadline, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = gemm::sdesc_sw128(sA + stage * A_BYTES);
          const uint64_t bdesc = gemm::sdesc_sw128(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            tc_mma_f8f6f4(tmem_base + buf * BN, adesc + 2ull * k, bdesc + 2ull * k, idesc, k != 0);
          tc_commit(&empty[stage]);
          tc_commit(&acc_full[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // every MMA this thread issued has completed before TMEM is released
      tc_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, globaltimer_ns() + 200000000ull, &no_abort);
    }
  }
  } else {
    if constexpr (EPI == 0) asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory");
    // ---------------- epilogue warps: promotion of every K block, then the tile's epilogue
    const int q = warp & 3;                   // TMEM lane quarter this warp may access
    const int half = (warp - EPI_BASE) >> 2;  // which half of the tile's columns
    const int row_in_tile = q * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    const int NB = p.N / 128;  // 128-row weight blocks per expert
    // this thread's two 64-column groups inside the 256-column accumulator
    const int col0 = EPI == 0 ? 64 * half : 128 * half;
    const int col1 = EPI == 0 ? 128 + 64 * half : 128 * half + 64;
    uint32_t it = 0, tcount = 0;
    bool ok = true;
    for (uint32_t tq = 0; ok; ++tq, ++tcount) {
      const int qi = tq % TILE_Q;
      if (!mbar_wait(&tq_full[qi], (tq / TILE_Q) & 1u, deadline, abort_flag)) break;
      const int tile = s_tile[qi];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tq_empty[qi]);
      if (tile < 0) break;
      int e, m_blk, n_t;
      gemm::decode_tile(s_mstart, P, NT, tile, e, m_blk, n_t);
      const int64_t row = (int64_t)m_blk * BM + row_in_tile;
      const bool valid = p.row_tok[row] >= 0;
      const int nb0 = EPI == 0 ? n_t : 2 * n_t + half;
      const int nb1 = EPI == 0 ? NB / 2 + n_t : 2 * n_t + half;
      const float* sb0 = p.sb + ((int64_t)e * NB + nb0) * KT;
      const float* sb1 = p.sb + ((int64_t)e * NB + nb1) * KT;
      float acc0[64], acc1[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        acc0[i] = 0.f;
        acc1[i] = 0.f;
      }
      // the next K block's activation scale (GEMM1: and weight scales) is loaded one step ahead
      float sa_next = p.sa[row], b0_next = 0.f, b1_next = 0.f;
      if constexpr (EPI == 0) {
        b0_next = __ldg(sb0);
        b1_next = __ldg(sb1);
      }
      for (int kt = 0; kt < KT; ++kt, ++it) {
        float f0, f1;
        if constexpr (EPI == 0) {
          f0 = sa_next * b0_next;
          f1 = sa_next * b1_next;
          if (kt + 1 < KT) {
            sa_next = p.sa[(int64_t)(kt + 1) * p.m_cap + row];
            b0_next = __ldg(sb0 + kt + 1);
            b1_next = __ldg(sb1 + kt + 1);
          }
        } else {
          const float sa = sa_next;
          if (kt + 1 < KT) sa_next = p.sa[(int64_t)(kt + 1) * p.m_cap + row];
          f0 = sa * __ldg(sb0 + kt);
          f1 = sa * __ldg(sb1 + kt);
        }
        const uint32_t buf = it & 1u;
        if (!mbar_wait(&acc_full[buf], (it >> 1) & 1u, deadline, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = t_lane + buf * BN;
        if constexpr (EPI == 0) {  // two TMEM loads in flight per wait (the register split leaves room)
          uint32_t va[32], vb[32];
          tmem_ld_32x32b_x32(tb + col0, va);
          tmem_ld_32x32b_x32(tb + col0 + 32, vb);
          tmem_wait_ld();
          fma32_pairs(acc0, va, f0);
          fma32_pairs(acc0 + 32, vb, f0);
          tmem_ld_32x32b_x32(tb + col1, va);
          tmem_ld_32x32b_x32(tb + col1 + 32, vb);
          tmem_wait_ld();
          tc_fence_before();  // this warp's reads of the buffer are complete: hand it back to the MMA warp
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
          fma32_pairs(acc1, va, f1);
          fma32_pairs(acc1 + 32, vb, f1);
        } else {
          uint32_t v[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld_32x32b_x32(tb + col0 + 32 * c, v);
            tmem_wait_ld();
            fma32_pairs(acc0 + 32 * c, v, f0);
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld_32x32b_x32(tb + col1 + 32 * c, v);
            tmem_wait_ld();
            if (c == 1) {  // this warp's reads of the buffer are complete: hand it back to the MMA warp
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[buf]);
            }
            fma32_pairs(acc1 + 32 * c, v, f1);
          }
        }
      }
      if (!ok) break;
      if constexpr (EPI == 0) {
        const int I = p.N / 2;
        const float lim = p.swiglu_limit;
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          float gv = acc0[i], uv = acc1[i];
          if (lim > 0.f) {
            gv = fminf(gv, lim);
            uv = fminf(fmaxf(uv, -lim), lim);
          }
          acc0[i] = gemm::silu_f(gv) * uv;
          amax = fmaxf(amax, fabsf(acc0[i]));
        }
        // the row's other 64 h values live in the partner warp (same lane quarter, other half)
        const uint32_t par = tcount & 1u;
        s_amax[(par * 2 + half) * 128 + row_in_tile] = amax;
        mbar_arrive(&amax_bar[q * 2 + par]);
        if (!mbar_wait(&amax_bar[q * 2 + par], (tcount >> 1) & 1u, deadline, abort_flag)) break;
        amax = fmaxf(amax, s_amax[(par * 2 + (half ^ 1)) * 128 + row_in_tile]);
        if (valid) {
          const float amax_c = fmaxf(amax, 1e-10f);
          const float scale = amax_c / kE4M3Max, inv = kE4M3Max / amax_c;
          uint4* dst = reinterpret_cast<uint4*>(p.out_q + row * I + n_t * 128 + half * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float* h = acc0 + 16 * j;
            dst[j] = make_uint4(e4m3x4(h[0], h[1], h[2], h[3], inv), e4m3x4(h[4], h[5], h[6], h[7], inv),
                                e4m3x4(h[8], h[9], h[10], h[11], inv), e4m3x4(h[12], h[13], h[14], h[15], inv));
          }
          if (half == 0) p.out_sa[(int64_t)n_t * p.m_cap + row] = scale;
        }
      } else {  // warp-cooperative stores through shared memory; every lane takes part, invalid rows masked
        const uint32_t valid_rows = __ballot_sync(0xffffffffu, valid);
        if (!valid_rows) continue;
        const float wr = valid ? p.row_w[row] : 0.f;
        uint8_t* wb = sOut + (warp - EPI_BASE) * 2048;
        __nv_bfloat16* out0 = p.out_bf + ((int64_t)m_blk * BM + q * 32) * p.N + (int64_t)n_t * BN + half * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float* a = c < 2 ? acc0 + 32 * c : acc1 + 32 * (c - 2);
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(a[2 * i] * wr, a[2 * i + 1] * wr);
            o[i] = *reinterpret_cast<const uint32_t*>(&b2);
          }
          gemm::store_rows_bf16x32(o, wb, out0 + c * 32, p.N, valid_rows, lane);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}
}  // namespace gemm8

// ------------------------------------------------------------------ FP8 activation quantisation + copy
// Every token once: bf16 row -> E4M3 codes + one fp32 scale per 128 values (scale = amax / 448, values multiplied
// by 448 / amax before the round-to-nearest-even, saturating conversion), stored straight into each of the token's
// local pair rows; the scales go to the K-block-major [H/128][m_cap] layout the GEMM epilogue reads.  One warp per
// token; each pass covers 256 values, a half-warp per 128-value block.
__global__ void __launch_bounds__(256) quant_permute_fp8_kernel(const __grid_constant__ QuantArgs p) {
  if (!p.desc->valid) return;
  const int n = p.desc->n;
  const int lane = threadIdx.x & 31;
  const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int H = p.H;
  float* dsf = reinterpret_cast<float*>(p.xq_sf);
  for (int64_t t = gwarp; t < n; t += nwarps) {
    const int32_t mine = lane < p.topk ? p.pair_pos[t * p.topk + lane] : -1;
    const uint32_t vmask = __ballot_sync(0xffffffffu, mine >= 0);
    if (!vmask) continue;
    int64_t local;
    const int r = row_of_token(p.desc, t, local);
    const __nv_bfloat16* src = p.x[r] + local * H;
    for (int base = 0; base < H; base += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + base + lane * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
      float v[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float amax_c = fmaxf(amax, 1e-10f);
      const float inv = gemm8::kE4M3Max / amax_c, scale = amax_c / gemm8::kE4M3Max;
      const uint2 codes = make_uint2(gemm8::e4m3x4(v[0], v[1], v[2], v[3], inv),
                                     gemm8::e4m3x4(v[4], v[5], v[6], v[7], inv));
      const int64_t kb = base / 128 + (lane >> 4);
      for (uint32_t m = vmask; m; m &= m - 1) {
        const int32_t row = __shfl_sync(0xffffffffu, mine, __ffs(m) - 1);
        *reinterpret_cast<uint2*>(p.xq + (int64_t)row * H + base + lane * 8) = codes;
        if ((lane & 15) == 0) dsf[kb * p.m_cap + row] = scale;
      }
    }
  }
}
