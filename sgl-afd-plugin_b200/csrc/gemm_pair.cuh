// K4/K5 on CTA pairs: the MXFP8 x MXFP4 grouped GEMMs of moe_gemm_kernel with one tcgen05 MMA spanning the two
// SMs of a thread-block cluster (.cta_group::2).  Included by ffn.cu (gemm::Params, decode helpers, epilogue).
//
// A pair tile is 256 rows (two 128-row blocks of one expert, one per CTA) x 256 columns.  Each CTA loads its own
// 128 activation rows and half (128 rows) of the tile's weight rows; the MMA reads the other half of B from the
// peer's shared memory, so a CTA stages 32 KB per 128-deep K step instead of 48 KB and the pipeline is 6 steps
// deep instead of 4.  Each CTA keeps the full 256 weight rows' scale atoms (1 KB) and its own activation scales.
//
// Roles (both CTAs run warps 0 and 2..9; warp 1 issues MMAs in the leader, rank 0, only):
//   warp 0    TMA producer: waits on its own `empty[s]`; the leader arms the leader's `full[s]` for both CTAs'
//             bytes; every load of either CTA completes on the leader's `full[s]`.  Each CTA loads only into its
//             own shared memory: no load is multicast.
//   warp 1    leader: scale copies into both CTAs' TMEM, 4 pair MMAs per K step, commit of each step to both
//             CTAs' `empty[s]` and of each tile to both CTAs' `acc_full`.  Both CTAs: TMEM alloc / dealloc.
//   warps 2-9 epilogue of the CTA's own 128 rows, same math as moe_gemm_kernel; TMEM is handed back by an arrive
//             on the leader's `acc_empty` (16 arrivals: both CTAs' epilogue warps).
// An expert with an odd number of blocks leaves the follower's half of its last pair tile without rows: the
// follower then loads the leader's block again (every access in bounds) and stores nothing.
// Every mbarrier wait is bounded by the job's deadline (an expired one raises the CTA's abort flag and reports
// ASAP_ST_PIPELINE_TIMEOUT).  The two cluster barriers (after set-up, before TMEM is freed) cannot be bounded;
// both CTAs reach each of them after bounded work only, and the early return for weights-as-M jobs is taken by
// both CTAs alike (it reads the same job descriptor).

namespace gemmP {
using gemm::BK;
using gemm::BM;
using gemm::BN;
constexpr int STAGES = 6;
constexpr int A_BYTES = BM * BK;          // this CTA's 128 activation rows, E4M3
constexpr int B_BYTES = (BN / 2) * BK;    // this CTA's 128 weight rows as the MMA reads them
constexpr int B_TX = (BN / 2) * BK / 2;   // their packed global bytes
constexpr int SFA_BYTES = 512, SFB_BYTES = 1024;
constexpr uint32_t CTA_TX = A_BYTES + B_TX + SFA_BYTES + SFB_BYTES;  // one CTA's bytes per K step
constexpr int NUM_EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + NUM_EPI_WARPS);
constexpr uint32_t TMEM_COLS = 512, TMEM_ACC = 0, TMEM_SFA = 256, TMEM_SFB = TMEM_SFA + 4 * STAGES;
static_assert(TMEM_SFB + 8 * STAGES <= TMEM_COLS, "scale-factor columns exceed TMEM");
constexpr int SMEM_TILES = STAGES * (A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES);
constexpr int STAGE_OUT_BYTES = NUM_EPI_WARPS * 2048;
constexpr int SMEM_BYTES = 1024 /*align slack*/ + SMEM_TILES + STAGE_OUT_BYTES + 1024 /*barriers*/ +
                           4 * (2 * ASAP_MAX_LOCAL_EXPERTS + 16);
static_assert(SMEM_BYTES <= 232448, "shared memory over the 227 KB per block");

// Tile -> expert e, leader block blk0 (the follower's is blk0 + 1), the expert's block count, n-tile.  Tiles run
// pair-fastest within (expert, n-tile), like moe_gemm_kernel's block-fastest order.
__device__ __forceinline__ void decode_pair(const int32_t* s_mstart, const int32_t* s_pstart, int P, int NT, int tile,
                                            int& e, int& blk0, int& nblk, int& n_t) {
  const int v = tile / NT;
  int lo = 0, hi = P;  // first index with pstart > v, minus one
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (s_pstart[mid] <= v) lo = mid + 1;
    else hi = mid;
  }
  e = lo - 1;
  const int pe = s_pstart[e + 1] - s_pstart[e];
  const int local = tile - NT * s_pstart[e];
  n_t = local / pe;
  blk0 = s_mstart[e] + 2 * (local % pe);
  nblk = s_mstart[e + 1] - s_mstart[e];
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1) moe_gemm_pair_kernel(const __grid_constant__ gemm::Params p) {
  if (p.desc->valid && p.desc->small) return;  // the weights-as-M kernel runs this job (same in both CTAs)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  uint8_t* sOut = sSFB + STAGES * SFB_BYTES;  // [NUM_EPI_WARPS][2048] output staging
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + STAGE_OUT_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* mma_done = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_mstart = reinterpret_cast<int32_t*>(tmem_slot + 4);
  int32_t* s_pstart = s_mstart + ASAP_MAX_LOCAL_EXPERTS + 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: leader (MMA issuer)
  const bool leader = rank == 0;
  const int P = p.P;
  const bool valid_job = p.desc->valid != 0;
  for (int i = threadIdx.x; i <= P; i += THREADS) s_mstart[i] = valid_job ? p.mstart[i] : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * NUM_EPI_WARPS);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmap_a);
    prefetch_tmap(&p.tmap_b);
    prefetch_tmap(&p.tmap_sfa);
    prefetch_tmap(&p.tmap_sfb);
  }
  __syncthreads();
  if (warp == 0) {  // pair-tile prefix over experts: pstart[e] = sum of ceil(blocks / 2) before e
    const int per = (P + 31) / 32;
    const int e0 = lane * per, e1 = min(e0 + per, P);
    int sum = 0;
    for (int e = e0; e < e1; ++e) sum += (s_mstart[e + 1] - s_mstart[e] + 1) >> 1;
    int incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += t;
    }
    int run = incl - sum;
    for (int e = e0; e < e1; ++e) {
      s_pstart[e] = run;
      run += (s_mstart[e + 1] - s_mstart[e] + 1) >> 1;
    }
    if (lane == 31) s_pstart[P] = incl;
  }
  // barriers initialised and TMEM allocated in both CTAs before any signal crosses to the peer
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int NT = p.N / BN, KT = p.K / BK;
  const int num_tiles = s_pstart[P] * NT;
  const int first = (int)cluster_id_x(), stride = (int)num_clusters_x();
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = first; tile < num_tiles && ok; tile += stride) {
        int e, blk0, nblk, n_t;
        decode_pair(s_mstart, s_pstart, P, NT, tile, e, blk0, nblk, n_t);
        const int m_blk = blk0 + ((int)rank < nblk - (blk0 - s_mstart[e]) ? (int)rank : 0);
        const int a_row = m_blk * BM;
        const int b_row = e * p.N + n_t * BN + (int)rank * (BN / 2);
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, deadline, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * CTA_TX);
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sA + stage * A_BYTES, &p.tmap_a, kt * BK, a_row, bar);
          tma_load_2d_pair(sB + stage * B_BYTES, &p.tmap_b, kt * BK, b_row, bar);
          tma_load_2d_pair(sSFA + stage * SFA_BYTES, &p.tmap_sfa, 0, m_blk * KT + kt, bar);
          tma_load_2d_pair(sSFB + stage * SFB_BYTES, &p.tmap_sfb, n_t * (SFB_BYTES / 4), e * KT + kt, bar);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: no copy into this CTA may still be in flight when it exits.  The leader waits for its last armed
      // stages to complete (they count both CTAs' bytes); the follower, whose copies complete on the leader's
      // barriers, waits for the MMA's release of those stages, which follows their completion.
      {
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
          mbar_wait(leader ? &full[s] : &empty[s], ph, drain_deadline, &no_abort);
        }
      }
      if (!ok) report(p.status, status_word(ASAP_ST_PIPELINE_TIMEOUT, 0, 0, EPI));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      const uint32_t idesc = gemm::idesc_mxf8f6f4(2 * BM, BN);
      bool ok = true;
      for (int tile = first; tile < num_tiles && ok; tile += stride) {
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
          const uint32_t t_sfa = tmem_base + TMEM_SFA + 4 * stage, t_sfb = tmem_base + TMEM_SFB + 8 * stage;
          tc_cp_pair_32x128b_warpx4(t_sfa, gemm::sdesc_sf(sSFA + stage * SFA_BYTES));
          tc_cp_pair_32x128b_warpx4(t_sfb, gemm::sdesc_sf(sSFB + stage * SFB_BYTES));
          tc_cp_pair_32x128b_warpx4(t_sfb + 4, gemm::sdesc_sf(sSFB + stage * SFB_BYTES + 512));
          const uint64_t adesc = gemm::sdesc_sw128(sA + stage * A_BYTES);
          const uint64_t bdesc = gemm::sdesc_sw128(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint32_t id = idesc | ((uint32_t)k << 29) | ((uint32_t)k << 4);
            tc_mma_pair_mxf8f6f4(tmem_base + TMEM_ACC, adesc + 2ull * k, bdesc + 2ull * k, id, (kt | k) != 0,
                                 t_sfa | ((uint32_t)k << 30), t_sfb | ((uint32_t)k << 30));
          }
          tc_commit_pair_all(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair_all(acc_full, 0x3);
        acc_phase ^= 1u;
      }
      // every MMA has completed (both CTAs' TMEM and shared memory are no longer read) before the teardown
      tc_commit_pair(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, globaltimer_ns() + 200000000ull, &no_abort);
      if (!ok) report(p.status, status_word(ASAP_ST_PIPELINE_TIMEOUT, 0, 1, EPI));
    }
  } else {
    // ---------------- epilogue warps (both CTAs, each its own 128 rows)
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which half of the tile's columns
    const int row_in_tile = q * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(acc_empty), 0);
    uint32_t acc_phase = 0;
    for (int tile = first; tile < num_tiles; tile += stride) {
      int e, blk0, nblk, n_t;
      decode_pair(s_mstart, s_pstart, P, NT, tile, e, blk0, nblk, n_t);
      const bool mine = (int)rank < nblk - (blk0 - s_mstart[e]);  // this CTA's half holds rows of expert e
      const int m_blk = mine ? blk0 + (int)rank : blk0;
      const int64_t row = (int64_t)m_blk * BM + row_in_tile;
      const bool valid = mine && p.row_tok[row] >= 0;
      if (!mbar_wait(acc_full, acc_phase, deadline, abort_flag)) break;
      tc_fence_after();
      uint32_t v[4][32];
      if constexpr (EPI == 0) {  // gate cols [64h, 64h+64) and the matching up cols 128 further
        tmem_ld_32x32b_x32(t_lane + TMEM_ACC + half * 64, v[0]);
        tmem_ld_32x32b_x32(t_lane + TMEM_ACC + half * 64 + 32, v[1]);
        tmem_ld_32x32b_x32(t_lane + TMEM_ACC + 128 + half * 64, v[2]);
        tmem_ld_32x32b_x32(t_lane + TMEM_ACC + 128 + half * 64 + 32, v[3]);
      } else {  // output cols [128h, 128h+128)
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_lane + TMEM_ACC + half * 128 + c * 32, v[c]);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
      acc_phase ^= 1u;
      gemm::epilogue_store<EPI>(p, v, row, valid, m_blk, n_t, q, half, sOut + (warp - 2) * 2048, lane);
    }
  }
  // Teardown: the leader's MMAs are complete and both CTAs' copies have landed (drains above); after the cluster
  // barrier no signal crosses between the CTAs, and both free their TMEM columns.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}
}  // namespace gemmP
