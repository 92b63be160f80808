// Small-segment grouped GEMMs (MXFP8 activations x MXFP4 weights) with the weights as the MMA's M operand:
// D[weight row][token] = W x X^T.  A tile is one 128-row weight block (GEMM1: the gate block and its up block)
// against one 128-row block of an expert's tokens; the MMA's N is 64 when at most 64 of those token rows are real,
// else 128, so a job whose experts hold a few rows each spends half (or less) of the tensor work the 128 x 256
// token-major tiles would spend on padding, while loading exactly the same weight and activation bytes per FLOP.
// Selected per workspace (asap_ffn_set_small_mode; per job on the device with mode -1, JobDesc.small set by the
// permutation's scan when the 128-row blocks are on average less than half full); the token-major kernels and these
// exit at once when the job is not theirs.  On B200 this variant measured slower than the token-major tiles for
// config 5's small jobs (GEMM1 0.30 vs 0.23 ms, GEMM2 0.18 vs 0.13 ms per F rank at T=1024), so it is opt-in.
// Included by ffn.cu (JobDesc, sf_atom_off, gemm:: helpers).

namespace gemmT {
constexpr int BW = 128, BT = 128, BK = 128;  // weight rows, token rows, K per stage
constexpr int STAGES = 4;
constexpr int W_BYTES = BW * BK;      // one weight block as the MMA reads it (16 bytes per 16 E2M1 values)
constexpr int W_TX = BW * BK / 2;     // its packed global bytes
constexpr int X_BYTES = BT * BK;      // activation block, E4M3
constexpr int SFW_BYTES = 1024, SFX_BYTES = 512;
constexpr int NUM_EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + NUM_EPI_WARPS);
// TMEM: gate accumulator [0, 128), up accumulator [128, 256) (GEMM2 uses the first), then per stage the weight
// scale columns (8) and the activation scale columns (4).
constexpr uint32_t TMEM_COLS = 512, TMEM_SFW = 256, TMEM_SFX = TMEM_SFW + 8 * STAGES;
static_assert(TMEM_SFX + 4 * STAGES <= TMEM_COLS, "scale-factor columns exceed TMEM");
constexpr int SMEM_TILES = STAGES * (2 * W_BYTES + X_BYTES + SFW_BYTES + SFX_BYTES);
constexpr int SMEM_BYTES = 1024 /*align slack*/ + SMEM_TILES + 1024 /*barriers*/ + 8 * (ASAP_MAX_LOCAL_EXPERTS + 8);
static_assert(SMEM_BYTES <= 232448, "shared memory over the 227 KB per block");

constexpr int PREFETCH = 8;  // K steps ahead the weight tiles are prefetched into L2 (small jobs stream weights from DRAM)

// L2 prefetch of one tensor tile (no shared memory, no completion tracking).
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(x), "r"(y)
               : "memory");
}

// kind::mxf8f6f4 block-scaled: A = E2M1 (weights), B = E4M3 (activations), UE8M0 scales, M x N.
__host__ __device__ constexpr uint32_t idesc_w4x8(int M, int N) {
  return (5u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) | ((uint32_t)(M >> 4) << 24);
}

struct Params {
  CUtensorMap tmap_w;  // weights [P * N, K] E2M1, 128-row boxes
  CUtensorMap tmap_x;  // activations [m_cap, K] E4M3, 128-row boxes
  const uint8_t* sfw;  // weight scale atoms per expert [K/128][N/128][512]
  uint64_t sfw_expert_stride;
  const uint8_t* sfx;  // activation scale atoms [m_cap/128][K/128][512]
  const JobDesc* desc;
  const int32_t* mstart;   // [P + 1] in 128-row blocks
  const int32_t* ecnt;     // [P] rows (pairs) per local expert
  const int32_t* row_tok;  // [m_cap]
  const float* row_w;      // [m_cap]
  uint8_t* out_q;          // GEMM1: [m_cap, N/2] E4M3
  uint8_t* out_sf;         // GEMM1: scale atoms [m_cap/128][(N/2)/128][512]
  __nv_bfloat16* out_bf;   // GEMM2: [m_cap, N]
  int32_t P, N, K;
  float swiglu_limit;
  uint64_t status, timeout_ns;
};

// A unit is two 128-row weight blocks (256 rows), accumulated side by side in TMEM [0, 128) and [128, 256).
// EPI 0 (GEMM1, N = 2I in the interleaved device layout): unit u = gate block u + up block u, epilogue
// h = silu(gate) * up quantised to MXFP8 (a warp's 32 lanes are one 32-feature scale block).
// EPI 1 (GEMM2, N = H): unit u = weight rows [256u, 256u + 256), epilogue bf16(acc * w[row]).
template <int EPI>
__global__ void __launch_bounds__(THREADS, 1) moe_gemm_t_kernel(const __grid_constant__ Params p) {
  if (!p.desc->valid || !p.desc->small) return;  // not this job's GEMM: leave before touching TMEM or barriers
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;                          // [STAGES][2][W_BYTES]
  uint8_t* sX = sW + STAGES * 2 * W_BYTES;     // [STAGES][X_BYTES]
  uint8_t* sSFW = sX + STAGES * X_BYTES;       // [STAGES][1024]
  uint8_t* sSFX = sSFW + STAGES * SFW_BYTES;   // [STAGES][512]
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFX + STAGES * SFX_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* mma_done = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_mstart = reinterpret_cast<int32_t*>(tmem_slot + 4);
  int32_t* s_ecnt = s_mstart + ASAP_MAX_LOCAL_EXPERTS + 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = p.P;
  for (int i = threadIdx.x; i <= P; i += THREADS) {
    s_mstart[i] = p.mstart[i];
    if (i < P) s_ecnt[i] = p.ecnt[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, NUM_EPI_WARPS);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmap_w);
    prefetch_tmap(&p.tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int NB = p.N / BW;                        // weight blocks per expert
  const int NU = NB / 2;                          // tile units (two weight blocks) per expert
  const int KT = p.K / BK;
  constexpr int nblk = 2;                         // weight blocks per unit
  const int num_tiles = s_mstart[P] * NU;
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      const uint64_t sfw_kstride = (uint64_t)NB * 512;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int e, m_blk, u;
        gemm::decode_tile(s_mstart, P, NU, tile, e, m_blk, u);
        const int w_row = e * p.N + u * BW * nblk;
        const uint8_t* sfw = p.sfw + (uint64_t)e * p.sfw_expert_stride + (uint64_t)u * nblk * 512;
        const uint8_t* sfx = p.sfx + (uint64_t)m_blk * KT * SFX_BYTES;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, deadline, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], (uint32_t)(nblk * (W_TX + 512) + X_BYTES + SFX_BYTES));
          // keep the weight stream PREFETCH steps ahead in L2 (at a tile's first step, the steps up to it too)
          for (int ka = kt == 0 ? 1 : kt + PREFETCH; ka <= kt + PREFETCH && ka < KT; ++ka)
            for (int b = 0; b < nblk; ++b) tma_prefetch_2d(&p.tmap_w, ka * BK, w_row + b * BW);
          for (int b = 0; b < nblk; ++b)
            tma_load_2d(sW + (stage * 2 + b) * W_BYTES, &p.tmap_w, kt * BK, w_row + b * BW, &full[stage]);
          tma_load_2d(sX + stage * X_BYTES, &p.tmap_x, kt * BK, m_blk * BT, &full[stage]);
          bulk_load(sSFW + stage * SFW_BYTES, sfw + (uint64_t)kt * sfw_kstride, (uint32_t)(nblk * 512), &full[stage]);
          bulk_load(sSFX + stage * SFX_BYTES, sfx + (uint64_t)kt * SFX_BYTES, SFX_BYTES, &full[stage]);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
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
      if (!ok) report(p.status, status_word(ASAP_ST_PIPELINE_TIMEOUT, 0, 0, 16 + EPI));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int e, m_blk, u;
        gemm::decode_tile(s_mstart, P, NU, tile, e, m_blk, u);
        const int real = s_ecnt[e] - (m_blk - s_mstart[e]) * BT;  // token rows of this block that hold a pair
        const int n_mma = real <= 64 ? 64 : 128;
        const uint32_t idesc = idesc_w4x8(BW, n_mma);
        if (!mbar_wait(acc_empty, acc_phase ^ 1u, deadline, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&full[stage], phase, deadline, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t t_sfw = tmem_base + TMEM_SFW + 8 * stage, t_sfx = tmem_base + TMEM_SFX + 4 * stage;
          for (int b = 0; b < nblk; ++b)
            tc_cp_32x128b_warpx4(t_sfw + 4 * b, gemm::sdesc_sf(sSFW + stage * SFW_BYTES + 512 * b));
          tc_cp_32x128b_warpx4(t_sfx, gemm::sdesc_sf(sSFX + stage * SFX_BYTES));
          const uint64_t xdesc = gemm::sdesc_sw128(sX + stage * X_BYTES);
          for (int b = 0; b < nblk; ++b) {
            const uint64_t wdesc = gemm::sdesc_sw128(sW + (stage * 2 + b) * W_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 32; ++k) {
              const uint32_t id = idesc | ((uint32_t)k << 29) | ((uint32_t)k << 4);
              tc_mma_mxf8f6f4(tmem_base + 128 * b, wdesc + 2ull * k, xdesc + 2ull * k, id, (kt | k) != 0,
                              (t_sfw + 4 * b) | ((uint32_t)k << 30), t_sfx | ((uint32_t)k << 30));
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(acc_full);
        acc_phase ^= 1u;
      }
      tc_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, globaltimer_ns() + 200000000ull, &no_abort);
    }
  } else {
    // ---------------- epilogue warps: lane = weight row (feature), columns = tokens
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int e, m_blk, u;
      gemm::decode_tile(s_mstart, P, NU, tile, e, m_blk, u);
      const int real = s_ecnt[e] - (m_blk - s_mstart[e]) * BT;
      const int n_mma = real <= 64 ? 64 : 128;
      const int cols = n_mma / 2;       // token columns of this warp: [half * cols, half * cols + cols)
      const int c0 = half * cols;
      if (!mbar_wait(acc_full, acc_phase, deadline, abort_flag)) break;
      tc_fence_after();
      uint32_t v[4][32];  // [block 0 (gate): 0..1 | block 1 (up): 2..3][32 columns]
      tmem_ld_32x32b_x32(t_lane + c0, v[0]);
      if (cols == 64) tmem_ld_32x32b_x32(t_lane + c0 + 32, v[1]);
      tmem_ld_32x32b_x32(t_lane + 128 + c0, v[2]);
      if (cols == 64) tmem_ld_32x32b_x32(t_lane + 128 + c0 + 32, v[3]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      acc_phase ^= 1u;
      const int64_t row0 = (int64_t)m_blk * BT + c0;
      const int feat = (EPI == 0 ? u * BW : u * 2 * BW) + q * 32 + lane;  // GEMM1: h feature; GEMM2: block 0's
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        if (ch * 32 >= cols) break;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = ch * 32 + i;  // column inside this warp's range (warp-uniform)
          const int64_t row = row0 + c;
          const bool valid = c0 + c < real && p.row_tok[row] >= 0;
          if constexpr (EPI == 0) {
            const int I = p.N / 2;
            float g = __uint_as_float(v[ch][i]), uu = __uint_as_float(v[2 + ch][i]);
            const float lim = p.swiglu_limit;
            if (lim > 0.f) {
              g = fminf(g, lim);
              uu = fminf(fmaxf(uu, -lim), lim);
            }
            const float h = gemm::silu_f(g) * uu;
            const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(h))));
            const uint32_t sb = mx_e4m3_scale_byte(amax);
            const uint32_t code = cvt_e4m3x2(h * mx_inv_scale(sb), 0.f) & 0xffu;
            if (valid) {
              p.out_q[row * I + feat] = (uint8_t)code;
              if (lane == 0) p.out_sf[sf_atom_off(row, (u * BW + q * 32) / 32, I / 32)] = (uint8_t)sb;
            }
          } else {
            if (valid) {
              const float wr = p.row_w[row];
              p.out_bf[row * p.N + feat] = __float2bfloat16_rn(__uint_as_float(v[ch][i]) * wr);
              p.out_bf[row * p.N + feat + BW] = __float2bfloat16_rn(__uint_as_float(v[2 + ch][i]) * wr);
            }
          }
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
}  // namespace gemmT
