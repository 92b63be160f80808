// libasap F side: doorbell waits (one message, several joined messages, or the first ready one), the expert-major
// permutation, activation quantisation (MXFP8, or FP8 per 1x128 for block-FP8 experts), the tcgen05 grouped GEMMs
// with fused epilogues (MXFP8 x MXFP4 block-scaled here; FP8 x FP8 with block-scale promotion in gemm_fp8.cuh;
// the weighted reduce that
// writes the replies straight into the A ranks' ResultArenas, and the CUDA-graph capture of whole jobs.
//
// Reference behaviour replaced here (python/sgl_asap_plugin/):
//   transport/server.py:262-320     FfnServer.poll/_row        -> ffn_wait_kernel (device-side doorbell spin)
//   srt/managers/scheduler.py:387-450 run_job / rows_of        -> asap_ffn_job (launch chain, arena views)
//   SGLang FusedMoE -> FlashInfer trtllm_fp4_block_scale_routed_moe (scheduler.py:410-412;
//   srt/layers/quantization/mxfp4_flashinfer_trtllm_moe.py:68-99)
//                                                              -> route_count/scan/place, quant_permute, moe_gemm<0,1>
//                                                                 (FP8: moe_gemm_fp8<0,1>), finalize_reply kernels
//   transport/server.py:340-350     FfnServer.reply            -> finalize_reply epilogue (P2P rows + done flag)
#include <cuda.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace asap {

int sm_count();

// ------------------------------------------------------------------ job descriptor and workspace layout
struct JobDesc {
  int32_t n, layer, epoch, valid;
  uint32_t seq;
  uint32_t sync;     // arrive counter of the finalize grid
  uint64_t t_seen;   // globaltimer (ns) when the doorbell wait saw the message (0: posted by the host)
  uint64_t t_reply;  // globaltimer (ns) when the reply's done flag was released
  int32_t rows;      // messages joined in this job (RowState entries after the descriptor)
  uint32_t tiles[2];  // next unclaimed tile of GEMM1 / GEMM2 (the GEMMs' dynamic tile scheduler), zeroed per job
  uint32_t pad[3];
};
static_assert(sizeof(JobDesc) == 64, "JobDesc is one cache line");

// A job answers up to kMaxJobRows messages at once (rows of several A replicas for the same layer and slot, as the
// reference's Job joins the Rows of a group, transport/server.py:322-337): tokens are numbered across the rows in
// row order; each row's state follows the descriptor in the workspace.
constexpr int kMaxJobRows = ASAP_MAX_JOB_ROWS;
struct RowState {
  int32_t n, off;  // tokens of this message and its first job-wide token index
  uint32_t seq;
  int32_t layer;
  int32_t view;    // which of the job's row views (x / ids / w / reply target) holds this message
  int32_t pad[3];
};
static_assert(sizeof(RowState) == 32, "RowState is 32 bytes");
__device__ __forceinline__ const RowState* row_states(const JobDesc* d) {
  return reinterpret_cast<const RowState*>(d + 1);
}
// The row view holding job-wide token t, and t's index inside that message.
__device__ __forceinline__ int row_of_token(const JobDesc* d, int64_t t, int64_t& local) {
  const RowState* rs = row_states(d);
  const int rows = d->rows;
  int r = 0;
  for (int i = 1; i < rows; ++i)
    if (t >= rs[i].off) r = i;
  local = t - rs[r].off;
  return rs[r].view;
}

constexpr int kPermChunks = 128;  // chunks of pairs the permutation is split into (upper bound)

struct WsLayout {
  int32_t n_max, topk, P, H, I;
  int64_t m_cap;  // rows of the expert-major activation buffers (multiple of 128)
  uint64_t desc, ecnt, mstart, hist, pair_pos, row_tok, row_w, ids_all, w_all, xq, xq_sf, hq, hq_sf, y2, total;
};

static WsLayout ws_layout(int n_max, int topk, int P, int H, int I) {
  WsLayout L;
  L.n_max = n_max;
  L.topk = topk;
  L.P = P;
  L.H = H;
  L.I = I;
  L.m_cap = align_up((uint64_t)n_max * topk + 128ull * P, 128);
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    uint64_t at = off;
    off = align_up(off + bytes, 1024);
    return at;
  };
  L.desc = take(sizeof(JobDesc) + sizeof(RowState) * kMaxJobRows);
  L.ecnt = take(4ull * ASAP_MAX_LOCAL_EXPERTS);
  L.mstart = take(4ull * (ASAP_MAX_LOCAL_EXPERTS + 1));
  L.hist = take(4ull * kPermChunks * ASAP_MAX_LOCAL_EXPERTS);
  L.pair_pos = take(4ull * n_max * topk);
  L.row_tok = take(4ull * L.m_cap);
  L.row_w = take(4ull * L.m_cap);
  L.ids_all = take(4ull * n_max * topk);  // ids / weights of a multi-row job, gathered in token order
  L.w_all = take(4ull * n_max * topk);
  L.xq = take((uint64_t)L.m_cap * H);
  L.xq_sf = take((uint64_t)L.m_cap * (H / 32));
  L.hq = take((uint64_t)L.m_cap * I);
  L.hq_sf = take((uint64_t)L.m_cap * (I / 32));
  L.y2 = take((uint64_t)L.m_cap * H * 2);
  L.total = off;
  return L;
}

// Byte offset of the E8M0 scale of (row r, 32-element block kb) inside a scale-factor atom array laid out
// [r / 128][kb / 4][512 B], the 512-byte atom holding 128 rows x 4 blocks as the tcgen05 scale-factor copy
// (32x128b.warpx4) reads it: byte (r % 32) * 16 + ((r / 32) % 4) * 4 + kb % 4.
__host__ __device__ __forceinline__ uint64_t sf_atom_off(int64_t r, int kb, int kblocks) {
  return ((uint64_t)(r >> 7) * (uint64_t)(kblocks >> 2) + (uint64_t)(kb >> 2)) * 512ull + (uint64_t)(r & 31) * 16ull +
         (uint64_t)((r >> 5) & 3) * 4ull + (uint64_t)(kb & 3);
}

// ------------------------------------------------------------------ K3: doorbell wait / host post
struct WaitArgs {
  JobDesc* d;
  int32_t rows, n_max, capacity;  // messages to wait for; tokens per message; tokens per job (workspace)
  const uint64_t* bell[kMaxJobRows];
  uint32_t last_seq[kMaxJobRows];
  uint32_t* seq_state[kMaxJobRows];  // device words holding the last consumed seq (used and advanced when set)
  int32_t epoch[kMaxJobRows];
  int32_t* any;  // non-NULL: answer ONE message, the first ready in round-robin order after *any (then updated)
  int32_t rest;  // answer every row not yet answered this round: rows whose seq word reached round_seq are left out
  uint32_t round_seq[kMaxJobRows];
  uint64_t status, timeout_ns;
};

// One warp; lane r spins (bounded) on row r's doorbell until its seq is cyclically ahead of last_seq[r], then
// decodes it.  The job is valid when every doorbell came, every epoch and size checks, all rows name the same
// layer and the tokens fit the workspace.  In the `rest` form a row whose sequence word already reached its
// round_seq (answered this round by an earlier job) is left out: the job joins the other rows' messages, its row
// states numbered in row order with the row as their view, and a job left with no row is empty (not valid, no
// error).
__global__ void ffn_wait_kernel(const __grid_constant__ WaitArgs a) {
  JobDesc* d = a.d;
  RowState* rs = reinterpret_cast<RowState*>(d + 1);
  const int lane = threadIdx.x;
  int ok = 1, n = 0, layer = 0, epoch = 0;
  uint32_t seq = 0;
  bool take = lane < a.rows;
  uint32_t last = 0;
  if (take) {
    last = a.seq_state[lane] ? *a.seq_state[lane] : a.last_seq[lane];
    if (a.rest && (int32_t)(last - a.round_seq[lane]) >= 0) take = false;  // answered this round already
  }
  if (take) {
    const uint64_t deadline = globaltimer_ns() + a.timeout_ns;
    uint64_t word = 0;
    for (;;) {
      word = ld_relaxed_sys_u64(a.bell[lane]);
      if ((int32_t)((uint32_t)word - last) > 0) break;
      if (globaltimer_ns() > deadline) {
        report(a.status, status_word(ASAP_ST_DOORBELL_TIMEOUT, lane, 0, last + 1u));
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    seq = (uint32_t)word;
    n = (int32_t)((word >> 32) & kMaxTokens);
    layer = (int32_t)((word >> 49) & kMaxLayer);
    epoch = (int32_t)(word >> 59);
    if (ok && a.seq_state[lane]) *a.seq_state[lane] = seq;  // consumed (a replayed graph waits for the next one)
    if (ok && (epoch != a.epoch[lane] || n < 1 || n > a.n_max)) {
      report(a.status, status_word(ASAP_ST_BAD_DOORBELL, lane, 0, seq));
      ok = 0;
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  const uint32_t taken = __ballot_sync(0xffffffffu, take);
  const int first = taken ? __ffs(taken) - 1 : 0;
  const int layer0 = __shfl_sync(0xffffffffu, layer, first);
  const bool same_layer = __all_sync(0xffffffffu, !take || layer == layer0);
  int incl = (ok && take) ? n : 0;  // inclusive scan of the taken rows' sizes
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  if (take)
    rs[__popc(taken & ((1u << lane) - 1u))] = RowState{ok ? n : 0, incl - (ok ? n : 0), seq, layer, lane, {0, 0, 0}};
  const uint32_t seq0 = __shfl_sync(0xffffffffu, seq, first);
  const int epoch0 = __shfl_sync(0xffffffffu, epoch, first);
  if (lane == 0) {
    d->t_seen = globaltimer_ns();
    d->t_reply = 0;
    d->tiles[0] = d->tiles[1] = 0;
    d->seq = seq0;
    d->layer = layer0;
    d->epoch = epoch0;
    d->sync = 0;
    d->rows = __popc(taken);
    bool valid = ok != 0 && taken != 0;
    if (valid && (!same_layer || total > a.capacity)) {
      report(a.status, status_word(ASAP_ST_BAD_JOB, 0, 0, seq0));
      valid = false;
    }
    d->n = valid ? total : 0;
    d->valid = valid ? 1 : 0;
  }
}

// Round-robin form (the reference's FfnServer.poll order over ready doorbells, transport/server.py:270-275): lane
// r polls row r's doorbell; the first ready row after the last answered one (*a.any) is taken, consumed through
// its sequence word and described as the job's only row.  Bounded like the all-rows wait.
__global__ void ffn_wait_any_kernel(const __grid_constant__ WaitArgs a) {
  JobDesc* d = a.d;
  RowState* rs = reinterpret_cast<RowState*>(d + 1);
  const int lane = threadIdx.x;
  const int rows = a.rows;
  const uint32_t last = lane < rows ? *a.seq_state[lane] : 0u;
  const int start = (*a.any + 1) % rows;
  const uint64_t deadline = globaltimer_ns() + a.timeout_ns;
  uint64_t word = 0;
  int pick = -1;
  for (;;) {
    bool ready = false;
    if (lane < rows) {
      word = ld_relaxed_sys_u64(a.bell[lane]);
      ready = (int32_t)((uint32_t)word - last) > 0;
    }
    const uint32_t mask = __ballot_sync(0xffffffffu, ready);
    if (mask) {  // rotate so that bit 0 is row `start`, take the lowest set bit
      const uint32_t full = rows >= 32 ? 0xffffffffu : ((1u << rows) - 1u);
      const uint32_t rot = ((mask >> start) | (mask << ((rows - start) & 31))) & full;
      pick = (start + __ffs(rot) - 1) % rows;
      break;
    }
    // lane 0's clock decides, so that the whole warp leaves the loop together (the ballot above needs all lanes)
    if (__shfl_sync(0xffffffffu, (int)(globaltimer_ns() > deadline), 0)) break;
    __nanosleep(64);
  }
  if (lane == 0) {
    d->t_seen = globaltimer_ns();
    d->t_reply = 0;
    d->tiles[0] = d->tiles[1] = 0;
    d->sync = 0;
    d->rows = 1;
  }
  if (pick < 0) {
    if (lane == 0) {
      report(a.status, status_word(ASAP_ST_DOORBELL_TIMEOUT, 0, 0, 0));
      d->valid = 0;
      d->n = 0;
    }
    return;
  }
  if (lane == pick) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    const uint32_t seq = (uint32_t)word;
    const int32_t n = (int32_t)((word >> 32) & kMaxTokens);
    const int32_t layer = (int32_t)((word >> 49) & kMaxLayer);
    const int32_t epoch = (int32_t)(word >> 59);
    *a.seq_state[lane] = seq;
    *a.any = lane;
    const bool valid = epoch == a.epoch[lane] && n >= 1 && n <= a.n_max && n <= a.capacity;
    if (!valid) report(a.status, status_word(ASAP_ST_BAD_DOORBELL, lane, 0, seq));
    rs[0] = RowState{valid ? n : 0, 0, seq, layer, lane, {0, 0, 0}};
    d->seq = seq;
    d->layer = layer;
    d->epoch = epoch;
    d->n = valid ? n : 0;
    __threadfence_block();
    d->valid = valid ? 1 : 0;
  }
}

struct PostArgs {
  JobDesc* d;
  int32_t rows, layer;
  uint32_t seq[kMaxJobRows];
  int32_t n[kMaxJobRows], epoch[kMaxJobRows];
};

__global__ void ffn_post_kernel(const __grid_constant__ PostArgs a) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  JobDesc* d = a.d;
  RowState* rs = reinterpret_cast<RowState*>(d + 1);
  int off = 0;
  for (int r = 0; r < a.rows; ++r) {
    rs[r] = RowState{a.n[r], off, a.seq[r], a.layer, r, {0, 0, 0}};
    off += a.n[r];
  }
  d->seq = a.seq[0];
  d->n = off;
  d->layer = a.layer;
  d->epoch = a.epoch[0];
  d->sync = 0;
  d->t_seen = 0;
  d->t_reply = 0;
  d->tiles[0] = d->tiles[1] = 0;
  d->rows = a.rows;
  d->valid = 1;
}

// Multi-row jobs: the rows' ids and weights copied into job-wide [n, topk] arrays for the permutation.
struct GatherArgs {
  const JobDesc* desc;
  int32_t topk;
  const int32_t* ids[kMaxJobRows];
  const float* w[kMaxJobRows];
  int32_t* ids_all;
  float* w_all;
};

__global__ void __launch_bounds__(256) gather_rows_kernel(const __grid_constant__ GatherArgs p) {
  if (!p.desc->valid) return;
  const int64_t total = (int64_t)p.desc->n * p.topk;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    int64_t local;
    const int r = row_of_token(p.desc, q / p.topk, local);
    const int64_t src = local * p.topk + q % p.topk;
    p.ids_all[q] = p.ids[r][src];
    p.w_all[q] = p.w[r][src];
  }
}

// ------------------------------------------------------------------ K3b-1: expert-major permutation
// Stable counting sort of the (token, slot) pairs whose expert is local, by (expert, token, slot), over many
// CTAs: count (per-chunk histograms) -> scan (tile-aligned expert bases, per-chunk bases) -> place.  Each
// expert's rows start on a 128-row boundary (one GEMM M tile never mixes experts).

struct PermArgs {
  const JobDesc* desc;
  const int32_t* ids;  // [n, topk] in the RecvArena
  const float* w;      // [n, topk]
  int32_t topk, P, expert_base;
  int32_t* ecnt;      // [P]
  int32_t* mstart;    // [P + 1] first 128-row tile of every expert; mstart[P] = tiles in all
  int32_t* pair_pos;  // [n, topk]
  int32_t* row_tok;   // [m_cap]
  float* row_w;       // [m_cap]
  int32_t* hist;      // [kPermChunks][ASAP_MAX_LOCAL_EXPERTS] chunk histograms, then chunk bases
};

__device__ __forceinline__ void perm_chunking(const PermArgs& p, int64_t& total, int64_t& chunk, int& chunks) {
  const int n = p.desc->valid ? p.desc->n : 0;
  total = (int64_t)n * p.topk;
  chunk = ((total + kPermChunks - 1) / kPermChunks + 31) / 32 * 32;
  if (chunk < 32) chunk = 32;
  chunks = (int)((total + chunk - 1) / chunk);
}

__global__ void __launch_bounds__(256) route_count_kernel(const __grid_constant__ PermArgs p) {
  __shared__ int32_t h[ASAP_MAX_LOCAL_EXPERTS];
  int64_t total, chunk;
  int chunks;
  perm_chunking(p, total, chunk, chunks);
  if ((int)blockIdx.x >= chunks) return;
  for (int i = threadIdx.x; i < p.P; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t q0 = blockIdx.x * chunk, q1 = min(total, q0 + chunk);
  for (int64_t q = q0 + threadIdx.x; q < q1; q += blockDim.x) {
    const int e = p.ids[q] - p.expert_base;
    if (e >= 0 && e < p.P) atomicAdd(&h[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < p.P; i += blockDim.x) p.hist[(int64_t)blockIdx.x * ASAP_MAX_LOCAL_EXPERTS + i] = h[i];
}

// One CTA: every chunk histogram is staged in shared memory with coalesced loads (eight in flight per thread), each
// expert's thread (threads < P) sums its column and turns it into chunk bases in place, the tile-aligned expert
// starts come from a block scan, and the bases and the padding rows go out with coalesced stores (a warp per
// expert for the padding: one thread storing its expert's padding rows alone made every warp store touch 32 lines).
constexpr int kScanThreads = 1024;
constexpr int kScanSmemBytes = kPermChunks * ASAP_MAX_LOCAL_EXPERTS * 4;
__global__ void __launch_bounds__(kScanThreads) route_scan_kernel(const __grid_constant__ PermArgs p) {
  extern __shared__ int32_t sh[];  // [chunks][P]
  __shared__ int32_t wsum[ASAP_MAX_LOCAL_EXPERTS / 32];
  __shared__ int32_t pad_lo[ASAP_MAX_LOCAL_EXPERTS], pad_hi[ASAP_MAX_LOCAL_EXPERTS];
  int64_t total, chunk;
  int chunks;
  perm_chunking(p, total, chunk, chunks);
  const int P = p.P;
  const int cells = chunks * P;
  for (int i0 = threadIdx.x; i0 < cells; i0 += kScanThreads * 8) {  // eight loads in flight per thread
    int32_t t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kScanThreads;
      const int g = i / P;
      t[u] = i < cells ? p.hist[(int64_t)g * ASAP_MAX_LOCAL_EXPERTS + (i - g * P)] : 0;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + u * kScanThreads < cells) sh[i0 + u * kScanThreads] = t[u];
  }
  __syncthreads();
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  int32_t c = 0;
  if (e < P)
    for (int g = 0; g < chunks; ++g) c += sh[g * P + e];
  const int32_t tiles = (e < P) ? (c + 127) / 128 : 0;
  int32_t v = tiles;  // exclusive scan of tiles over experts (warps 0..7 hold experts 0..255)
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += u;
  }
  if (lane == 31 && warp < ASAP_MAX_LOCAL_EXPERTS / 32) wsum[warp] = v;
  __syncthreads();
  int32_t before = 0;
  for (int w = 0; w < warp && w < ASAP_MAX_LOCAL_EXPERTS / 32; ++w) before += wsum[w];
  const int32_t mst = before + v - tiles;
  if (e < P) {
    p.ecnt[e] = c;
    p.mstart[e] = mst;
    int32_t base = mst * 128;
    for (int g = 0; g < chunks; ++g) {  // chunk bases, in place
      const int32_t t = sh[g * P + e];
      sh[g * P + e] = base;
      base += t;
    }
    pad_lo[e] = base;  // padding rows of the expert's last tile: [base, (mst + tiles) * 128)
    pad_hi[e] = (mst + tiles) * 128;
    if (e == P - 1) p.mstart[P] = mst + tiles;
  }
  __syncthreads();
  for (int x = warp; x < P; x += kScanThreads / 32)  // padding rows: no token (a warp per expert, coalesced)
    for (int32_t r = pad_lo[x] + lane; r < pad_hi[x]; r += 32) {
      p.row_tok[r] = -1;
      p.row_w[r] = 0.f;
    }
  for (int i = threadIdx.x; i < cells; i += kScanThreads) {
    const int g = i / P, e2 = i - g * P;
    p.hist[(int64_t)g * ASAP_MAX_LOCAL_EXPERTS + e2] = sh[i];
  }
}

__global__ void __launch_bounds__(32) route_place_kernel(const __grid_constant__ PermArgs p) {
  __shared__ int32_t off[ASAP_MAX_LOCAL_EXPERTS];
  int64_t total, chunk;
  int chunks;
  perm_chunking(p, total, chunk, chunks);
  if ((int)blockIdx.x >= chunks) return;
  const int lane = threadIdx.x;
  for (int i = lane; i < p.P; i += 32) off[i] = p.hist[(int64_t)blockIdx.x * ASAP_MAX_LOCAL_EXPERTS + i];
  __syncwarp();
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int64_t q0 = blockIdx.x * chunk, q1 = min(total, q0 + chunk);
  constexpr int U = 8;  // 32-pair steps whose ids / weights are loaded together (one round trip per U steps)
  for (int64_t qs = q0; qs < q1; qs += 32 * U) {
    int eu[U];
    float wu[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t q = qs + 32 * u + lane;
      eu[u] = -1;
      wu[u] = 0.f;
      if (q < q1) {
        const int e = p.ids[q] - p.expert_base;
        eu[u] = (e >= 0 && e < p.P) ? e : -1;
        wu[u] = p.w[q];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {  // the steps in pair order: positions as with one step at a time
      const int64_t q = qs + 32 * u + lane;
      const int e = eu[u];
      const uint32_t active = __ballot_sync(0xffffffffu, e >= 0);
      const uint32_t peers = __match_any_sync(0xffffffffu, e) & active;
      int32_t pos = -1;
      if (e >= 0) pos = off[e] + __popc(peers & lt_mask);
      __syncwarp();
      if (e >= 0 && (peers & lt_mask) == 0) off[e] += __popc(peers);
      __syncwarp();
      if (q < q1) {
        p.pair_pos[q] = pos;
        if (pos >= 0) {
          p.row_tok[pos] = (int32_t)(q / p.topk);
          p.row_w[pos] = wu[u];
        }
      }
    }
  }
}

// ------------------------------------------------------------------ K3b-2: gather + MXFP8 quantisation
struct QuantArgs {
  const JobDesc* desc;
  int32_t H, topk;
  int64_t m_cap;
  const __nv_bfloat16* x[kMaxJobRows];  // [n_r, H] per message, in the RecvArena
  const int32_t* pair_pos;              // [n, topk] permuted row of each (token, slot), -1 when not local
  uint8_t* xq;                          // [m_cap, H] E4M3, expert-major
  uint8_t* xq_sf;                       // MXFP8: scale atoms [m_cap/128][H/128][512]; FP8: fp32 [H/128][m_cap]
};

// Quantise 32 consecutive fp32 values to E4M3 with one E8M0 scale; returns the scale byte.
__device__ __forceinline__ uint32_t mx_quant32(const float (&v)[32], uint4& lo, uint4& hi) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const uint32_t sb = mx_e4m3_scale_byte(amax);
  const float inv = mx_inv_scale(sb);
  uint32_t wv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t a = cvt_e4m3x2(v[4 * i] * inv, v[4 * i + 1] * inv);
    const uint32_t b = cvt_e4m3x2(v[4 * i + 2] * inv, v[4 * i + 3] * inv);
    wv[i] = a | (b << 16);
  }
  lo = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  hi = make_uint4(wv[4], wv[5], wv[6], wv[7]);
  return sb;
}

// Every token once: bf16 row -> E4M3 codes + one E8M0 scale per 32 values (OCP MX rule), stored straight into
// each of the token's local pair rows of the expert-major buffer (rows and scale atoms), so no intermediate
// per-token copy is written and read back.  One warp per token; lane L quantises the 32-value blocks L, L+32, ...
__global__ void __launch_bounds__(256) quant_permute_kernel(const __grid_constant__ QuantArgs p) {
  if (!p.desc->valid) return;
  const int n = p.desc->n;
  const int lane = threadIdx.x & 31;
  const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int H = p.H, kblocks = H / 32;
  for (int64_t t = gwarp; t < n; t += nwarps) {
    const int32_t mine = lane < p.topk ? p.pair_pos[t * p.topk + lane] : -1;
    const uint32_t vmask = __ballot_sync(0xffffffffu, mine >= 0);
    if (!vmask) continue;  // no local expert: nothing to copy
    int64_t local;
    const int r = row_of_token(p.desc, t, local);
    const uint4* src = reinterpret_cast<const uint4*>(p.x[r] + local * H);
    for (int kb0 = 0; kb0 < kblocks; kb0 += 32) {
      const int kb = kb0 + lane;
      const bool act = kb < kblocks;
      uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
      uint32_t sb = 0;
      if (act) {
        float v[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 u = src[kb * 4 + c];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            v[c * 8 + 2 * i] = f.x;
            v[c * 8 + 2 * i + 1] = f.y;
          }
        }
        sb = mx_quant32(v, lo, hi);
      }
      // the scale bytes of 4 consecutive blocks are 4 consecutive atom bytes: one word, stored by the group's
      // first lane (kblocks is a multiple of 4, so a group is all active or all inactive)
      const uint32_t word = sb | (__shfl_down_sync(0xffffffffu, sb, 1) << 8) |
                            (__shfl_down_sync(0xffffffffu, sb, 2) << 16) | (__shfl_down_sync(0xffffffffu, sb, 3) << 24);
      // codes regrouped so that each store instruction writes 512 contiguous bytes: in half h, lane j stores the
      // 16-byte unit j of blocks [kb0 + 16 h, kb0 + 16 h + 16) (block 16 h + j / 2, its low or high 16 bytes)
      uint4 unit[2];
      bool unit_act[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int src = 16 * h + (lane >> 1);
        const uint4 l2 = make_uint4(__shfl_sync(0xffffffffu, lo.x, src), __shfl_sync(0xffffffffu, lo.y, src),
                                    __shfl_sync(0xffffffffu, lo.z, src), __shfl_sync(0xffffffffu, lo.w, src));
        const uint4 h2 = make_uint4(__shfl_sync(0xffffffffu, hi.x, src), __shfl_sync(0xffffffffu, hi.y, src),
                                    __shfl_sync(0xffffffffu, hi.z, src), __shfl_sync(0xffffffffu, hi.w, src));
        unit[h] = (lane & 1) ? h2 : l2;
        unit_act[h] = kb0 + src < kblocks;
      }
      for (uint32_t m = vmask; m; m &= m - 1) {
        const int32_t row = __shfl_sync(0xffffffffu, mine, __ffs(m) - 1);
        uint4* dst = reinterpret_cast<uint4*>(p.xq + (int64_t)row * H + (int64_t)kb0 * 32);
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (unit_act[h]) dst[32 * h + lane] = unit[h];
        if (act && (lane & 3) == 0)
          *reinterpret_cast<uint32_t*>(p.xq_sf + sf_atom_off(row, kb, kblocks)) = word;
      }
    }
  }
}

// ------------------------------------------------------------------ K4/K5: grouped block-scaled GEMM
namespace gemm {
constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;        // E4M3 tile
constexpr int B_BYTES = BN * BK;        // E2M1 tile as the MMA reads it: 16 values per 16 bytes
constexpr int B_TX = BN * BK / 2;       // bytes the TMA moves for it (packed in global memory)
constexpr int SFA_BYTES = 512, SFB_BYTES = 1024;
constexpr uint32_t STAGE_TX = A_BYTES + B_TX + SFA_BYTES + SFB_BYTES;
constexpr int NUM_EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + NUM_EPI_WARPS);
// TMEM columns: the 256-column accumulator, then one set of scale-factor columns per pipeline stage (SFA 4,
// SFB 8), so the scale copy of stage s+1 never waits for the MMAs still reading stage s's scales.
constexpr uint32_t TMEM_COLS = 512, TMEM_ACC = 0, TMEM_SFA = 256, TMEM_SFB = TMEM_SFA + 4 * STAGES;
static_assert(TMEM_SFB + 8 * STAGES <= TMEM_COLS, "scale-factor columns exceed TMEM");
constexpr int SMEM_TILES = STAGES * (A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES);
constexpr int STAGE_OUT_BYTES = NUM_EPI_WARPS * 2048;  // per epilogue warp: 32 rows x 64 B of output in flight
// Tiles are handed out at run time: the producer claims the next tile index from the job's counter (so CTAs that
// start late -- beside another kernel on the GPU -- simply take fewer tiles) and passes it to the MMA and epilogue
// warps through a queue of TILE_Q entries in shared memory.
constexpr int TILE_Q = 8;
constexpr int SMEM_BYTES =
    1024 /*align slack*/ + SMEM_TILES + STAGE_OUT_BYTES + 1024 /*barriers*/ + 4 * (ASAP_MAX_LOCAL_EXPERTS + 8);
static_assert(SMEM_BYTES <= 232448, "shared memory over the 227 KB per block");

// tcgen05 instruction descriptor, kind::mxf8f6f4 block-scaled: A = E4M3, B = E2M1, both K-major,
// UE8M0 scales, M x N.  Scale-factor byte ids are OR-ed in per MMA.
__host__ __device__ constexpr uint32_t idesc_mxf8f6f4(int M, int N) {
  return (0u << 7) | (5u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row core groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_sw128(const void* p) {
  const uint64_t a = smem_u32(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// Descriptor of one 512-byte scale-factor atom (32 rows x 16 bytes, no swizzle) for tcgen05.cp.
__device__ __forceinline__ uint64_t sdesc_sf(const void* p) {
  const uint64_t a = smem_u32(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

struct Params {
  CUtensorMap tmap_a;  // activations [m_cap, K] bytes (E4M3)
  CUtensorMap tmap_b;  // weights [P * N, K] E2M1 (4-bit, unpacked to 16 B per 16 values in smem)
  const uint8_t* sfa;  // activation scale atoms [m_cap/128][K/128][512]
  const uint8_t* sfb;  // weight scale atoms per expert [K/128][N/128][512]
  uint64_t sfb_expert_stride;
  const JobDesc* desc;
  const int32_t* mstart;   // [P + 1]
  const int32_t* row_tok;  // [m_cap]
  const float* row_w;      // [m_cap]
  uint8_t* out_q;          // GEMM1: [m_cap, N/2] E4M3
  uint8_t* out_sf;         // GEMM1: scale atoms [m_cap/128][(N/2)/128][512]
  __nv_bfloat16* out_bf;   // GEMM2: [m_cap, N]
  uint32_t* tile_ctr;      // the job's tile counter of this GEMM (JobDesc::tiles)
  int32_t P, N, K;
  float swiglu_limit;
  uint64_t status, timeout_ns;
};

__device__ __forceinline__ void decode_tile(const int32_t* s_mstart, int P, int NT, int tile, int& e, int& m_blk,
                                            int& n_t) {
  const int v = tile / NT;  // lies in [mstart[e], mstart[e+1]) of its expert
  int lo = 0, hi = P;       // first index with mstart > v, minus one
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (s_mstart[mid] <= v) lo = mid + 1;
    else hi = mid;
  }
  e = lo - 1;
  const int mt = s_mstart[e + 1] - s_mstart[e];
  const int local = tile - NT * s_mstart[e];
  n_t = local / mt;
  m_blk = s_mstart[e] + local % mt;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + expf(-g)); }

// Store a warp's 32 rows x 32 bf16 (lane = row, o = its 32 values packed in pairs) through a 2 KB shared-memory
// buffer, so that every global store instruction writes 8 rows x 64 contiguous bytes instead of 32 rows x 16 B.
// 16-byte units are XOR-swizzled by (row >> 1) & 3: both the row-wise writes and the transposed reads touch each
// group of 4 banks 4 times (the minimum for 512 bytes).  Rows whose bit in `valid` is clear are not stored.
__device__ __forceinline__ void store_rows_bf16x32(const uint32_t (&o)[16], uint8_t* wb, __nv_bfloat16* out0,
                                                   int64_t row_stride, uint32_t valid, int lane) {
  uint4* mine = reinterpret_cast<uint4*>(wb + lane * 64);
#pragma unroll
  for (int u = 0; u < 4; ++u) mine[u ^ ((lane >> 1) & 3)] = make_uint4(o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = i * 8 + (lane >> 2), u = lane & 3;
    const uint4 val = reinterpret_cast<const uint4*>(wb + row * 64)[u ^ ((row >> 1) & 3)];
    if ((valid >> row) & 1u) *reinterpret_cast<uint4*>(out0 + row * row_stride + u * 8) = val;
  }
  __syncwarp();
}

// One epilogue warp's share of a finished 128 x 256 accumulator tile, already drained from TMEM into v: lane = row
// `row` of quarter q, column half `half`.  EPI 0: h = silu(gate) * up quantised to MXFP8 (gate columns
// [64 half, 64 half + 64) of the tile, up columns 128 further).  EPI 1: bf16(acc * w[row]) through the warp's 2 KB
// staging buffer `wb`.
template <int EPI>
__device__ __forceinline__ void epilogue_store(const Params& p, const uint32_t (&v)[4][32], int64_t row, bool valid,
                                               int m_blk, int n_t, int q, int half, uint8_t* wb, int lane) {
  if constexpr (EPI == 1) {  // warp-cooperative stores: every lane takes part, invalid rows are masked
    const uint32_t valid_rows = __ballot_sync(0xffffffffu, valid);
    if (!valid_rows) return;
    const float wr = valid ? p.row_w[row] : 0.f;
    __nv_bfloat16* out0 = p.out_bf + ((int64_t)m_blk * BM + q * 32) * p.N + (int64_t)n_t * BN + half * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const __nv_bfloat162 b2 =
            __floats2bfloat162_rn(__uint_as_float(v[c][2 * i]) * wr, __uint_as_float(v[c][2 * i + 1]) * wr);
        o[i] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      store_rows_bf16x32(o, wb, out0 + c * 32, p.N, valid_rows, lane);
    }
  } else {
    if (!valid) return;
    const int I = p.N / 2;
    const int kblocks = I / 32;
    const float lim = p.swiglu_limit;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float h[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float gv = __uint_as_float(v[c][i]), uv = __uint_as_float(v[2 + c][i]);
        if (lim > 0.f) {
          gv = fminf(gv, lim);
          uv = fminf(fmaxf(uv, -lim), lim);
        }
        h[i] = silu_f(gv) * uv;
      }
      uint4 lo, hi;
      const uint32_t sb = mx_quant32(h, lo, hi);
      const int hcol = n_t * 128 + half * 64 + c * 32;
      uint4* dst = reinterpret_cast<uint4*>(p.out_q + row * I + hcol);
      dst[0] = lo;
      dst[1] = hi;
      p.out_sf[sf_atom_off(row, hcol / 32, kblocks)] = (uint8_t)sb;
    }
  }
}

// EPI 0: h = silu(gate) * up, quantised to MXFP8 (GEMM1).  EPI 1: bf16(acc * w[row]) (GEMM2).
template <int EPI>
__global__ void __launch_bounds__(THREADS, 1) moe_gemm_kernel(const __grid_constant__ Params p) {
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
  uint64_t* tq_full = mma_done + 1;     // [TILE_Q] a tile index was published
  uint64_t* tq_empty = tq_full + TILE_Q;  // [TILE_Q] the MMA warp and every epilogue warp have read it
  int32_t* s_tile = reinterpret_cast<int32_t*>(tq_empty + TILE_Q);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_tile + TILE_Q);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_mstart = reinterpret_cast<int32_t*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = p.P;
  const bool valid_job = p.desc->valid != 0;
  for (int i = threadIdx.x; i <= P; i += THREADS) s_mstart[i] = valid_job ? p.mstart[i] : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, NUM_EPI_WARPS);
    mbar_init(mma_done, 1);
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
        decode_tile(s_mstart, P, NT, tile, e, m_blk, n_t);
        const int a_row = m_blk * BM;
        const int b_row = e * p.N + n_t * BN;
        const uint8_t* sfa = p.sfa + (uint64_t)m_blk * KT * SFA_BYTES;
        const uint8_t* sfb = p.sfb + (uint64_t)e * p.sfb_expert_stride + (uint64_t)n_t * SFB_BYTES;
        const uint64_t sfb_kstride = (uint64_t)(p.N / 128) * 512;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, deadline, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_TX);
          tma_load_2d(sA + stage * A_BYTES, &p.tmap_a, kt * BK, a_row, &full[stage]);
          tma_load_2d(sB + stage * B_BYTES, &p.tmap_b, kt * BK, b_row, &full[stage]);
          bulk_load(sSFA + stage * SFA_BYTES, sfa + (uint64_t)kt * SFA_BYTES, SFA_BYTES, &full[stage]);
          bulk_load(sSFB + stage * SFB_BYTES, sfb + (uint64_t)kt * sfb_kstride, SFB_BYTES, &full[stage]);
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
      if (!ok) report(p.status, status_word(ASAP_ST_PIPELINE_TIMEOUT, 0, 0, EPI));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      const uint32_t idesc = idesc_mxf8f6f4(BM, BN);
      bool ok = true;
      for (uint32_t tq = 0; ok; ++tq) {
        const int q = tq % TILE_Q;
        if (!mbar_wait(&tq_full[q], (tq / TILE_Q) & 1u, deadline, abort_flag)) break;
        const int tile = s_tile[q];
        mbar_arrive(&tq_empty[q]);
        if (tile < 0) break;
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
          tc_cp_32x128b_warpx4(t_sfa, sdesc_sf(sSFA + stage * SFA_BYTES));
          tc_cp_32x128b_warpx4(t_sfb, sdesc_sf(sSFB + stage * SFB_BYTES));
          tc_cp_32x128b_warpx4(t_sfb + 4, sdesc_sf(sSFB + stage * SFB_BYTES + 512));
          const uint64_t adesc = sdesc_sw128(sA + stage * A_BYTES);
          const uint64_t bdesc = sdesc_sw128(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint32_t id = idesc | ((uint32_t)k << 29) | ((uint32_t)k << 4);
            tc_mma_mxf8f6f4(tmem_base + TMEM_ACC, adesc + 2ull * k, bdesc + 2ull * k, id, (kt | k) != 0,
                            t_sfa | ((uint32_t)k << 30), t_sfb | ((uint32_t)k << 30));
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
      // every MMA this thread issued has completed before TMEM is released
      tc_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, globaltimer_ns() + 200000000ull, &no_abort);
    }
  } else {
    // ---------------- epilogue warps
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;   // which half of the tile's columns
    const int row_in_tile = q * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    uint32_t acc_phase = 0;
    for (uint32_t tq = 0;; ++tq) {
      const int qi = tq % TILE_Q;
      if (!mbar_wait(&tq_full[qi], (tq / TILE_Q) & 1u, deadline, abort_flag)) break;
      const int tile = s_tile[qi];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tq_empty[qi]);
      if (tile < 0) break;
      int e, m_blk, n_t;
      decode_tile(s_mstart, P, NT, tile, e, m_blk, n_t);
      const int64_t row = (int64_t)m_blk * BM + row_in_tile;
      const bool valid = p.row_tok[row] >= 0;
      if (!mbar_wait(acc_full, acc_phase, deadline, abort_flag)) break;
      tc_fence_after();
      // Drain this warp's slice of the accumulator into registers and hand TMEM back at once: the MMA warp
      // starts the next tile while this warp does the epilogue math and stores.
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
      if (lane == 0) mbar_arrive(acc_empty);
      acc_phase ^= 1u;
      epilogue_store<EPI>(p, v, row, valid, m_blk, n_t, q, half, sOut + (warp - 2) * 2048, lane);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}
}  // namespace gemm

#include "gemm_fp8.cuh"

// ------------------------------------------------------------------ K5b: weighted reduce + reply
struct FinalArgs {
  const JobDesc* desc;
  int32_t topk, H;
  const int32_t* pair_pos;    // [n, topk]
  const __nv_bfloat16* y2;    // [m_cap, H], rows already weighted
  __nv_bfloat16* reply_seg[kMaxJobRows];  // each message's A ResultArena seg(f, slot) (peer memory across GPUs)
  uint32_t* reply_done[kMaxJobRows];      // each message's done flag (f, slot); NULL: no flag
  JobDesc* desc_rw;
};

__global__ void __launch_bounds__(256) finalize_reply_kernel(const __grid_constant__ FinalArgs p) {
  if (!p.desc->valid) return;
  const int n = p.desc->n;
  const int lane = threadIdx.x & 31;
  const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int H = p.H, nvec = H / 8;
  for (int64_t t = gwarp; t < n; t += nwarps) {
    int64_t local;
    const int row = row_of_token(p.desc, t, local);
    __nv_bfloat16* dst = p.reply_seg[row] + local * H;
    // this token's local pairs, in ascending slot order (the summation order)
    const int32_t mine = lane < p.topk ? p.pair_pos[t * p.topk + lane] : -1;
    const uint32_t vmask = __ballot_sync(0xffffffffu, mine >= 0);
    const int cnt = __popc(vmask);
    const __nv_bfloat16* rowp[8];  // the first 8 rows, resolved once per token
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int src = __fns(vmask, 0, i + 1);
      const int32_t pos = __shfl_sync(0xffffffffu, mine, src & 31);
      rowp[i] = p.y2 + (int64_t)(i < cnt ? pos : 0) * H;
    }
    int32_t extra[24];  // rows 8.. (more than 8 local experts of one token; cnt is warp-uniform)
    for (int i = 8; i < cnt; ++i) extra[i - 8] = __shfl_sync(0xffffffffu, mine, __fns(vmask, 0, i + 1) & 31);
    for (int c = lane; c < nvec; c += 32) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)  // all loads in flight, then the adds in slot order
        if (i < cnt) v[i] = *reinterpret_cast<const uint4*>(rowp[i] + (int64_t)c * 8);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i >= cnt) break;
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
      for (int i = 8; i < cnt; ++i) {  // more than 8 local experts of one token: the rest one by one
        const uint4 u = *reinterpret_cast<const uint4*>(p.y2 + (int64_t)extra[i - 8] * H + (int64_t)c * 8);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
      uint4 r;
      __nv_bfloat162* rh = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
      for (int i = 0; i < 4; ++i) rh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      *reinterpret_cast<uint4*>(dst + (int64_t)c * 8) = r;
    }
  }
  // Reply rows visible to A before its done flag (server.py:347-350 ordering).
  __syncthreads();
  __shared__ uint32_t last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = (atomicAdd(&p.desc_rw->sync, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    p.desc_rw->t_reply = globaltimer_ns();
    __threadfence_system();
    const RowState* rs = row_states(p.desc);
    for (int r = 0; r < p.desc->rows; ++r) {
      const int v = rs[r].view;
      if (p.reply_done[v]) st_release_sys_u32(p.reply_done[v], rs[r].seq);
    }
  }
}

// ------------------------------------------------------------------ host side: tensor maps, handles
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

static int make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                        uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, const char* what,
                        CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return ASAP_ECUDA;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled(%s) failed: %d", what, (int)r);
    return ASAP_ECUDA;
  }
  return ASAP_OK;
}

enum ExpertsKind { kMxfp4 = 0, kFp8Block = 1 };
struct ExpertsHandle {
  ExpertsKind kind;
  asap_mxfp4_experts_t e;   // kMxfp4 (num_local/expert_base/hidden/inter filled for both kinds)
  asap_fp8_experts_t f8;    // kFp8Block
  CUtensorMap w13_map, w2_map;
};
constexpr int kTimedKernels = 5;  // routing (count+scan+place), quantise+permute, gemm1, gemm2, finalize_reply
constexpr int kTimedJobs = 64;     // ring of event sets: the last 64 jobs since timing was enabled
struct WsHandle {
  uint8_t* base;
  WsLayout L;
  CUtensorMap xq_map, hq_map;
  bool timing = false;
  int jobs = 0;  // jobs recorded since enable
  cudaEvent_t ev[kTimedJobs][kTimedKernels + 1] = {};
  cudaEvent_t split = nullptr;  // GEMM2 done -> the reply stream's finalize (asap_ffn_job_rows_overlap)
};

static std::mutex g_mu;
static std::unordered_map<uint64_t, ExpertsHandle*> g_experts;
static std::unordered_map<uint64_t, WsHandle*> g_ws;
static uint64_t g_next = 1;

static ExpertsHandle* get_experts(uint64_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_experts.find(h);
  return it == g_experts.end() ? nullptr : it->second;
}
static WsHandle* get_ws(uint64_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_ws.find(h);
  return it == g_ws.end() ? nullptr : it->second;
}

static bool gemm_attr_set = false;

static int ensure_gemm_attrs() {
  if (gemm_attr_set) return ASAP_OK;
  ASAP_CUDA(cudaFuncSetAttribute(gemm::moe_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 gemm::SMEM_BYTES));
  ASAP_CUDA(cudaFuncSetAttribute(gemm::moe_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 gemm::SMEM_BYTES));
  ASAP_CUDA(cudaFuncSetAttribute(gemm8::moe_gemm_fp8_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 gemm8::SMEM_BYTES));
  ASAP_CUDA(cudaFuncSetAttribute(gemm8::moe_gemm_fp8_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 gemm8::SMEM_BYTES));
  ASAP_CUDA(cudaFuncSetAttribute(route_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kScanSmemBytes));
  gemm_attr_set = true;
  return ASAP_OK;
}

// K5b launch shared by both weight kinds, on `st` with `ctas` CTAs; `mark` records the job's last timing event.
template <class Mark>
static int finalize(JobDesc* desc, const WsLayout& L, const PermArgs& pa, uint8_t* B, int R,
                    const asap_ffn_row_t* rows, cudaStream_t st, int ctas, Mark& mark) {
  FinalArgs fa{};
  fa.desc = desc;
  fa.topk = L.topk;
  fa.H = L.H;
  fa.pair_pos = pa.pair_pos;
  fa.y2 = (const __nv_bfloat16*)(B + L.y2);
  for (int r = 0; r < R; ++r) {
    fa.reply_seg[r] = (__nv_bfloat16*)rows[r].reply_seg;
    fa.reply_done[r] = (uint32_t*)rows[r].reply_done;
  }
  fa.desc_rw = desc;
  finalize_reply_kernel<<<ctas, 256, 0, st>>>(fa);
  ASAP_CHECK_LAUNCH("finalize_reply_kernel");
  mark(5, st);
  return ASAP_OK;
}

}  // namespace asap

using namespace asap;

extern "C" {

int asap_experts_register(const asap_mxfp4_experts_t* e, uint64_t* handle) {
  if (!e || !handle) {
    set_error("asap_experts_register: NULL argument");
    return ASAP_EINVAL;
  }
  if (e->num_local < 1 || e->num_local > ASAP_MAX_LOCAL_EXPERTS || e->hidden % 256 || e->inter % 128 ||
      e->hidden <= 0 || e->inter <= 0 || e->expert_base < 0) {
    set_error("asap_experts_register: need 1 <= num_local <= %d, hidden %% 256 == 0, inter %% 128 == 0 (got %d, %d, %d)",
              ASAP_MAX_LOCAL_EXPERTS, e->num_local, e->hidden, e->inter);
    return ASAP_EINVAL;
  }
  if ((e->w13 & 31) || (e->w2 & 31) || (e->w13_sf & 15) || (e->w2_sf & 15) || !e->w13 || !e->w2 || !e->w13_sf ||
      !e->w2_sf) {
    set_error("asap_experts_register: weights must be 32-byte and scales 16-byte aligned, non-NULL");
    return ASAP_EINVAL;
  }
  ExpertsHandle* h = new ExpertsHandle;
  h->kind = kMxfp4;
  h->e = *e;
  const uint64_t P = e->num_local, H = e->hidden, I = e->inter;
  int rc = make_tmap_2d(&h->w13_map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, (const void*)e->w13, H, P * 2 * I, H / 2,
                        gemm::BK, gemm::BN, "w13");
  if (!rc)
    rc = make_tmap_2d(&h->w2_map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, (const void*)e->w2, I, P * H, I / 2, gemm::BK,
                      gemm::BN, "w2");
  if (rc) {
    delete h;
    return rc;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  *handle = g_next++;
  g_experts[*handle] = h;
  return ASAP_OK;
}

int asap_experts_register_fp8(const asap_fp8_experts_t* e, uint64_t* handle) {
  if (!e || !handle) {
    set_error("asap_experts_register_fp8: NULL argument");
    return ASAP_EINVAL;
  }
  if (e->num_local < 1 || e->num_local > ASAP_MAX_LOCAL_EXPERTS || e->hidden % 256 || e->inter % 128 ||
      e->hidden <= 0 || e->inter <= 0 || e->expert_base < 0) {
    set_error("asap_experts_register_fp8: need 1 <= num_local <= %d, hidden %% 256 == 0, inter %% 128 == 0 "
              "(got %d, %d, %d)",
              ASAP_MAX_LOCAL_EXPERTS, e->num_local, e->hidden, e->inter);
    return ASAP_EINVAL;
  }
  if ((e->w13 & 15) || (e->w2 & 15) || (e->w13_scale & 3) || (e->w2_scale & 3) || !e->w13 || !e->w2 ||
      !e->w13_scale || !e->w2_scale) {
    set_error("asap_experts_register_fp8: weights must be 16-byte and scales 4-byte aligned, non-NULL");
    return ASAP_EINVAL;
  }
  ExpertsHandle* h = new ExpertsHandle;
  h->kind = kFp8Block;
  h->f8 = *e;
  memset(&h->e, 0, sizeof(h->e));
  h->e.num_local = e->num_local;
  h->e.expert_base = e->expert_base;
  h->e.hidden = e->hidden;
  h->e.inter = e->inter;
  const uint64_t P = e->num_local, H = e->hidden, I = e->inter;
  int rc = make_tmap_2d(&h->w13_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (const void*)e->w13, H, P * 2 * I, H, gemm8::BK,
                        128, "w13 fp8");
  if (!rc)
    rc = make_tmap_2d(&h->w2_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (const void*)e->w2, I, P * H, I, gemm8::BK, 128,
                      "w2 fp8");
  if (rc) {
    delete h;
    return rc;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  *handle = g_next++;
  g_experts[*handle] = h;
  return ASAP_OK;
}

int asap_experts_release(uint64_t handle) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_experts.find(handle);
  if (it == g_experts.end()) {
    set_error("asap_experts_release: unknown handle");
    return ASAP_EINVAL;
  }
  delete it->second;
  g_experts.erase(it);
  return ASAP_OK;
}

uint64_t asap_ffn_ws_bytes(int32_t n_max, int32_t topk, int32_t num_local, int32_t hidden, int32_t inter) {
  if (n_max < 1 || topk < 1 || num_local < 1 || hidden < 1 || inter < 1) return 0;
  return ws_layout(n_max, topk, num_local, hidden, inter).total;
}

int asap_ffn_ws_register(uint64_t ws, int32_t n_max, int32_t topk, int32_t num_local, int32_t hidden,
                         int32_t inter, uint64_t* handle) {
  if (!ws || (ws & 1023) || !handle || n_max < 1 || topk < 1 || topk > 32 || num_local < 1 ||
      num_local > ASAP_MAX_LOCAL_EXPERTS || hidden % 256 || inter % 128 || hidden <= 0 || inter <= 0) {
    set_error("asap_ffn_ws_register: ws must be 1024-byte aligned; 1 <= topk <= 32, 1 <= num_local <= %d, "
              "hidden %% 256 == 0, inter %% 128 == 0",
              ASAP_MAX_LOCAL_EXPERTS);
    return ASAP_EINVAL;
  }
  // kernel attributes and the SM count are settled here, outside any stream capture of the jobs
  int arc = ensure_gemm_attrs();
  if (arc) return arc;
  (void)sm_count();
  WsHandle* h = new WsHandle;
  h->base = (uint8_t*)ws;
  h->L = ws_layout(n_max, topk, num_local, hidden, inter);
  int rc = make_tmap_2d(&h->xq_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, h->base + h->L.xq, hidden, h->L.m_cap, hidden,
                        gemm::BK, gemm::BM, "xq");
  if (!rc)
    rc = make_tmap_2d(&h->hq_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, h->base + h->L.hq, inter, h->L.m_cap, inter,
                      gemm::BK, gemm::BM, "hq");
  if (rc) {
    delete h;
    return rc;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  *handle = g_next++;
  g_ws[*handle] = h;
  return ASAP_OK;
}

int asap_ffn_ws_release(uint64_t handle) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_ws.find(handle);
  if (it == g_ws.end()) {
    set_error("asap_ffn_ws_release: unknown handle");
    return ASAP_EINVAL;
  }
  for (int j = 0; j < kTimedJobs; ++j)
    for (int i = 0; i <= kTimedKernels; ++i)
      if (it->second->ev[j][i]) cudaEventDestroy(it->second->ev[j][i]);
  if (it->second->split) cudaEventDestroy(it->second->split);
  delete it->second;
  g_ws.erase(it);
  return ASAP_OK;
}

static int ffn_wait_impl(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint32_t* last_seqs,
                         const uint64_t* seq_states, const int32_t* expect_epochs, int32_t n_max, uint64_t status,
                         uint64_t timeout_ns, void* stream, const uint32_t* round_seqs = nullptr) {
  WsHandle* w = get_ws(ws_handle);
  if (!w || rows < 1 || rows > kMaxJobRows || !bells || !(last_seqs || seq_states) || !expect_epochs) {
    set_error("asap_ffn_wait: unknown workspace handle, NULL arrays or rows %d outside [1, %d]", rows, kMaxJobRows);
    return ASAP_EINVAL;
  }
  if (n_max < 1 || n_max > w->L.n_max) {
    set_error("asap_ffn_wait: n_max %d outside the workspace's %d", n_max, w->L.n_max);
    return ASAP_EINVAL;
  }
  WaitArgs a{};
  a.d = (JobDesc*)(w->base + w->L.desc);
  a.rows = rows;
  a.n_max = n_max;
  a.capacity = w->L.n_max;
  for (int r = 0; r < rows; ++r) {
    if (!bells[r] || (bells[r] & 7)) {
      set_error("asap_ffn_wait: doorbell %d is NULL or misaligned", r);
      return ASAP_EINVAL;
    }
    if (seq_states && (!seq_states[r] || (seq_states[r] & 3))) {
      set_error("asap_ffn_wait: sequence state word %d is NULL or misaligned", r);
      return ASAP_EINVAL;
    }
    a.bell[r] = (const uint64_t*)bells[r];
    a.last_seq[r] = last_seqs ? last_seqs[r] : 0u;
    a.seq_state[r] = seq_states ? (uint32_t*)seq_states[r] : nullptr;
    a.epoch[r] = expect_epochs[r];
    a.round_seq[r] = round_seqs ? round_seqs[r] : 0u;
  }
  a.rest = round_seqs ? 1 : 0;
  a.status = status;
  a.timeout_ns = timeout_ns;
  ffn_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a);
  ASAP_CHECK_LAUNCH("ffn_wait_kernel");
  return ASAP_OK;
}

int asap_ffn_wait_rows(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint32_t* last_seqs,
                       const int32_t* expect_epochs, int32_t n_max, uint64_t status, uint64_t timeout_ns,
                       void* stream) {
  if (!last_seqs) {
    set_error("asap_ffn_wait: NULL last_seqs");
    return ASAP_EINVAL;
  }
  return ffn_wait_impl(ws_handle, rows, bells, last_seqs, nullptr, expect_epochs, n_max, status, timeout_ns, stream);
}

int asap_ffn_wait_state(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint64_t* seq_states,
                        const int32_t* expect_epochs, int32_t n_max, uint64_t status, uint64_t timeout_ns,
                        void* stream) {
  if (!seq_states) {
    set_error("asap_ffn_wait_state: NULL seq_states");
    return ASAP_EINVAL;
  }
  return ffn_wait_impl(ws_handle, rows, bells, nullptr, seq_states, expect_epochs, n_max, status, timeout_ns, stream);
}

int asap_ffn_wait_rest(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint64_t* seq_states,
                       const uint32_t* round_seqs, const int32_t* expect_epochs, int32_t n_max, uint64_t status,
                       uint64_t timeout_ns, void* stream) {
  if (!seq_states || !round_seqs) {
    set_error("asap_ffn_wait_rest: NULL seq_states or round_seqs");
    return ASAP_EINVAL;
  }
  return ffn_wait_impl(ws_handle, rows, bells, nullptr, seq_states, expect_epochs, n_max, status, timeout_ns, stream,
                       round_seqs);
}

int asap_ffn_wait_any(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint64_t* seq_states,
                      const int32_t* expect_epochs, int32_t n_max, uint64_t rr_state, uint64_t status,
                      uint64_t timeout_ns, void* stream) {
  WsHandle* w = get_ws(ws_handle);
  if (!w || rows < 1 || rows > kMaxJobRows || !bells || !seq_states || !expect_epochs || !rr_state ||
      (rr_state & 3)) {
    set_error("asap_ffn_wait_any: unknown workspace handle, NULL arrays / round-robin word or rows %d outside "
              "[1, %d]", rows, kMaxJobRows);
    return ASAP_EINVAL;
  }
  if (n_max < 1 || n_max > w->L.n_max) {
    set_error("asap_ffn_wait_any: n_max %d outside the workspace's %d", n_max, w->L.n_max);
    return ASAP_EINVAL;
  }
  WaitArgs a{};
  a.d = (JobDesc*)(w->base + w->L.desc);
  a.rows = rows;
  a.n_max = n_max;
  a.capacity = w->L.n_max;
  for (int r = 0; r < rows; ++r) {
    if (!bells[r] || (bells[r] & 7) || !seq_states[r] || (seq_states[r] & 3)) {
      set_error("asap_ffn_wait_any: doorbell or sequence word %d is NULL or misaligned", r);
      return ASAP_EINVAL;
    }
    a.bell[r] = (const uint64_t*)bells[r];
    a.seq_state[r] = (uint32_t*)seq_states[r];
    a.epoch[r] = expect_epochs[r];
  }
  a.any = (int32_t*)rr_state;
  a.status = status;
  a.timeout_ns = timeout_ns;
  ffn_wait_any_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a);
  ASAP_CHECK_LAUNCH("ffn_wait_any_kernel");
  return ASAP_OK;
}

int asap_ffn_wait(uint64_t ws_handle, uint64_t bell, uint32_t last_seq, int32_t expect_epoch, int32_t n_max,
                  uint64_t status, uint64_t timeout_ns, void* stream) {
  return asap_ffn_wait_rows(ws_handle, 1, &bell, &last_seq, &expect_epoch, n_max, status, timeout_ns, stream);
}

// ---------------------------------------------------------------- CUDA graphs of F chains
int asap_graph_begin(void* stream) {
  ASAP_CUDA(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal));
  return ASAP_OK;
}

int asap_graph_end(void* stream, uint64_t* graph) {
  if (!graph) {
    set_error("asap_graph_end: NULL graph");
    return ASAP_EINVAL;
  }
  cudaGraph_t g = nullptr;
  ASAP_CUDA(cudaStreamEndCapture((cudaStream_t)stream, &g));
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    set_error("cudaGraphInstantiate failed: %d %s", (int)e, cudaGetErrorString(e));
    return ASAP_ECUDA;
  }
  *graph = (uint64_t)exec;
  return ASAP_OK;
}

int asap_graph_launch(uint64_t graph, void* stream) {
  if (!graph) {
    set_error("asap_graph_launch: NULL graph");
    return ASAP_EINVAL;
  }
  ASAP_CUDA(cudaGraphLaunch((cudaGraphExec_t)graph, (cudaStream_t)stream));
  return ASAP_OK;
}

int asap_graph_release(uint64_t graph) {
  if (graph) ASAP_CUDA(cudaGraphExecDestroy((cudaGraphExec_t)graph));
  return ASAP_OK;
}

int asap_ffn_post_rows(uint64_t ws_handle, int32_t rows, const uint32_t* seqs, const int32_t* ns, int32_t layer_id,
                       const int32_t* epochs, void* stream) {
  WsHandle* w = get_ws(ws_handle);
  if (!w || rows < 1 || rows > kMaxJobRows || !seqs || !ns || !epochs) {
    set_error("asap_ffn_post: unknown workspace handle, NULL arrays or rows %d outside [1, %d]", rows, kMaxJobRows);
    return ASAP_EINVAL;
  }
  PostArgs a{};
  a.d = (JobDesc*)(w->base + w->L.desc);
  a.rows = rows;
  a.layer = layer_id;
  int64_t total = 0;
  for (int r = 0; r < rows; ++r) {
    if (ns[r] < 1) {
      set_error("asap_ffn_post: n_tokens %d of row %d below 1", ns[r], r);
      return ASAP_EINVAL;
    }
    total += ns[r];
    a.seq[r] = seqs[r];
    a.n[r] = ns[r];
    a.epoch[r] = epochs[r];
  }
  if (total > w->L.n_max) {
    set_error("asap_ffn_post: %lld tokens exceed the workspace's %d", (long long)total, w->L.n_max);
    return ASAP_EINVAL;
  }
  ffn_post_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a);
  ASAP_CHECK_LAUNCH("ffn_post_kernel");
  return ASAP_OK;
}

int asap_ffn_post(uint64_t ws_handle, uint32_t seq, int32_t n, int32_t layer_id, int32_t epoch, void* stream) {
  return asap_ffn_post_rows(ws_handle, 1, &seq, &n, layer_id, &epoch, stream);
}

int asap_ffn_job(uint64_t experts_handle, uint64_t ws_handle, uint64_t x, uint64_t ids, uint64_t w,
                 uint64_t reply_seg, uint64_t reply_done, float swiglu_limit, uint64_t status, uint64_t timeout_ns,
                 void* stream) {
  const asap_ffn_row_t row = {x, ids, w, reply_seg, reply_done};
  return asap_ffn_job_rows(experts_handle, ws_handle, 1, &row, swiglu_limit, status, timeout_ns, stream);
}

static int ffn_job_impl(uint64_t experts_handle, uint64_t ws_handle, int32_t R, const asap_ffn_row_t* rows,
                        float swiglu_limit, uint64_t status, uint64_t timeout_ns, cudaStream_t st,
                        cudaStream_t reply_st, int32_t gemm_ctas, int32_t reply_ctas) {
  ExpertsHandle* eh = get_experts(experts_handle);
  WsHandle* wh = get_ws(ws_handle);
  if (!eh || !wh) {
    set_error("asap_ffn_job: unknown experts or workspace handle");
    return ASAP_EINVAL;
  }
  const asap_mxfp4_experts_t& E = eh->e;
  const WsLayout& L = wh->L;
  if (E.num_local != L.P || E.hidden != L.H || E.inter != L.I) {
    set_error("asap_ffn_job: experts (P=%d H=%d I=%d) and workspace (P=%d H=%d I=%d) disagree", E.num_local,
              E.hidden, E.inter, L.P, L.H, L.I);
    return ASAP_EINVAL;
  }
  if (R < 1 || R > kMaxJobRows || !rows) {
    set_error("asap_ffn_job: rows %d outside [1, %d] or NULL", R, kMaxJobRows);
    return ASAP_EINVAL;
  }
  for (int r = 0; r < R; ++r) {
    const asap_ffn_row_t& q = rows[r];
    if (!q.x || !q.ids || !q.w || !q.reply_seg || (q.x & 15) || (q.reply_seg & 15) || (q.reply_done & 3) ||
        (q.ids & 3) || (q.w & 3)) {
      set_error("asap_ffn_job: row %d: x/reply_seg must be 16-byte aligned and non-NULL", r);
      return ASAP_EINVAL;
    }
  }
  int rc = ensure_gemm_attrs();
  if (rc) return rc;
  if (reply_st && !wh->split) ASAP_CUDA(cudaEventCreateWithFlags(&wh->split, cudaEventDisableTiming));
  uint8_t* B = wh->base;
  JobDesc* desc = (JobDesc*)(B + L.desc);
  const int sms = sm_count();
  const int gctas = gemm_ctas > 0 && gemm_ctas < sms ? gemm_ctas : sms;  // persistent GEMM grids

  PermArgs pa{};
  pa.desc = desc;
  pa.ids = R == 1 ? (const int32_t*)rows[0].ids : (const int32_t*)(B + L.ids_all);
  pa.w = R == 1 ? (const float*)rows[0].w : (const float*)(B + L.w_all);
  pa.topk = L.topk;
  pa.P = L.P;
  pa.expert_base = E.expert_base;
  pa.ecnt = (int32_t*)(B + L.ecnt);
  pa.mstart = (int32_t*)(B + L.mstart);
  pa.pair_pos = (int32_t*)(B + L.pair_pos);
  pa.row_tok = (int32_t*)(B + L.row_tok);
  pa.row_w = (float*)(B + L.row_w);
  pa.hist = (int32_t*)(B + L.hist);
  const int slot_ev = wh->jobs % kTimedJobs;
  if (wh->timing) ++wh->jobs;
  auto mark = [&](int i, cudaStream_t on) {
    if (wh->timing) cudaEventRecord(wh->ev[slot_ev][i], on);
  };
  // the reduce + reply: on `st` after GEMM2, or on `reply_st` (after an event) while `st` goes on to the next job
  auto reply = [&]() -> int {
    if (!reply_st) return finalize(desc, L, pa, B, R, rows, st, sms * 4, mark);
    ASAP_CUDA(cudaEventRecord(wh->split, st));
    ASAP_CUDA(cudaStreamWaitEvent(reply_st, wh->split, 0));
    return finalize(desc, L, pa, B, R, rows, reply_st, reply_ctas > 0 ? reply_ctas : sms * 4, mark);
  };
  mark(0, st);
  if (!pa.desc || !pa.ids || !pa.w || !pa.ecnt || !pa.mstart || !pa.pair_pos || !pa.row_tok || !pa.row_w ||
      !pa.hist) {
    set_error("asap_ffn_job: internal error, a permutation buffer is unset");
    return ASAP_EINVAL;
  }
  if (R > 1) {
    GatherArgs ga{};
    ga.desc = desc;
    ga.topk = L.topk;
    for (int r = 0; r < R; ++r) {
      ga.ids[r] = (const int32_t*)rows[r].ids;
      ga.w[r] = (const float*)rows[r].w;
    }
    ga.ids_all = (int32_t*)(B + L.ids_all);
    ga.w_all = (float*)(B + L.w_all);
    gather_rows_kernel<<<sms * 2, 256, 0, st>>>(ga);
    ASAP_CHECK_LAUNCH("gather_rows_kernel");
  }
  route_count_kernel<<<kPermChunks, 256, 0, st>>>(pa);
  ASAP_CHECK_LAUNCH("route_count_kernel");
  route_scan_kernel<<<1, kScanThreads, kScanSmemBytes, st>>>(pa);
  ASAP_CHECK_LAUNCH("route_scan_kernel");
  route_place_kernel<<<kPermChunks, 32, 0, st>>>(pa);
  ASAP_CHECK_LAUNCH("route_place_kernel");
  mark(1, st);

  QuantArgs qa{};
  qa.desc = desc;
  qa.H = L.H;
  qa.topk = L.topk;
  qa.m_cap = L.m_cap;
  for (int r = 0; r < R; ++r) qa.x[r] = (const __nv_bfloat16*)rows[r].x;
  qa.pair_pos = pa.pair_pos;
  qa.xq = B + L.xq;
  qa.xq_sf = B + L.xq_sf;
  if (eh->kind == kFp8Block) {
    quant_permute_fp8_kernel<<<sms * 4, 256, 0, st>>>(qa);
    ASAP_CHECK_LAUNCH("quant_permute_fp8_kernel");
    mark(2, st);
    gemm8::Params g1;
    memset(&g1, 0, sizeof(g1));
    g1.tmap_a = wh->xq_map;
    g1.tmap_b = eh->w13_map;
    g1.sa = (const float*)(B + L.xq_sf);
    g1.sb = (const float*)eh->f8.w13_scale;
    g1.m_cap = L.m_cap;
    g1.desc = desc;
    g1.mstart = pa.mstart;
    g1.row_tok = pa.row_tok;
    g1.row_w = pa.row_w;
    g1.out_q = B + L.hq;
    g1.out_sa = (float*)(B + L.hq_sf);
    g1.tile_ctr = &desc->tiles[0];
    g1.P = L.P;
    g1.N = 2 * L.I;
    g1.K = L.H;
    g1.swiglu_limit = swiglu_limit;
    g1.status = status;
    g1.timeout_ns = timeout_ns;
    gemm8::moe_gemm_fp8_kernel<0><<<gctas, gemm8::Cfg<0>::THREADS, gemm8::SMEM_BYTES, st>>>(g1);
    ASAP_CHECK_LAUNCH("moe_gemm_fp8_kernel<0>");
    mark(3, st);
    gemm8::Params g2 = g1;
    g2.tmap_a = wh->hq_map;
    g2.tmap_b = eh->w2_map;
    g2.sa = (const float*)(B + L.hq_sf);
    g2.sb = (const float*)eh->f8.w2_scale;
    g2.out_q = nullptr;
    g2.out_sa = nullptr;
    g2.out_bf = (__nv_bfloat16*)(B + L.y2);
    g2.tile_ctr = &desc->tiles[1];
    g2.N = L.H;
    g2.K = L.I;
    gemm8::moe_gemm_fp8_kernel<1><<<gctas, gemm8::Cfg<1>::THREADS, gemm8::SMEM_BYTES, st>>>(g2);
    ASAP_CHECK_LAUNCH("moe_gemm_fp8_kernel<1>");
    mark(4, st);
    return reply();
  }
  quant_permute_kernel<<<sms * 4, 256, 0, st>>>(qa);
  ASAP_CHECK_LAUNCH("quant_permute_kernel");
  mark(2, st);

  gemm::Params g1;
  memset(&g1, 0, sizeof(g1));
  g1.tmap_a = wh->xq_map;
  g1.tmap_b = eh->w13_map;
  g1.sfa = B + L.xq_sf;
  g1.sfb = (const uint8_t*)E.w13_sf;
  g1.sfb_expert_stride = (uint64_t)(L.H / 32) * (2 * L.I);
  g1.desc = desc;
  g1.mstart = pa.mstart;
  g1.row_tok = pa.row_tok;
  g1.row_w = pa.row_w;
  g1.out_q = B + L.hq;
  g1.out_sf = B + L.hq_sf;
  g1.tile_ctr = &desc->tiles[0];
  g1.P = L.P;
  g1.N = 2 * L.I;
  g1.K = L.H;
  g1.swiglu_limit = swiglu_limit;
  g1.status = status;
  g1.timeout_ns = timeout_ns;
  gemm::moe_gemm_kernel<0><<<gctas, gemm::THREADS, gemm::SMEM_BYTES, st>>>(g1);
  ASAP_CHECK_LAUNCH("moe_gemm_kernel<0>");
  mark(3, st);

  gemm::Params g2 = g1;
  g2.tmap_a = wh->hq_map;
  g2.tmap_b = eh->w2_map;
  g2.sfa = B + L.hq_sf;
  g2.sfb = (const uint8_t*)E.w2_sf;
  g2.sfb_expert_stride = (uint64_t)(L.I / 32) * L.H;
  g2.out_q = nullptr;
  g2.out_sf = nullptr;
  g2.out_bf = (__nv_bfloat16*)(B + L.y2);
  g2.tile_ctr = &desc->tiles[1];
  g2.N = L.H;
  g2.K = L.I;
  gemm::moe_gemm_kernel<1><<<gctas, gemm::THREADS, gemm::SMEM_BYTES, st>>>(g2);
  ASAP_CHECK_LAUNCH("moe_gemm_kernel<1>");
  mark(4, st);

  return reply();
}

int asap_ffn_job_rows(uint64_t experts_handle, uint64_t ws_handle, int32_t R, const asap_ffn_row_t* rows,
                      float swiglu_limit, uint64_t status, uint64_t timeout_ns, void* stream) {
  return ffn_job_impl(experts_handle, ws_handle, R, rows, swiglu_limit, status, timeout_ns, (cudaStream_t)stream,
                      nullptr, 0, 0);
}

int asap_ffn_job_rows_overlap(uint64_t experts_handle, uint64_t ws_handle, int32_t R, const asap_ffn_row_t* rows,
                              float swiglu_limit, uint64_t status, uint64_t timeout_ns, void* stream,
                              void* reply_stream, int32_t gemm_ctas, int32_t reply_ctas) {
  if (!reply_stream || reply_stream == stream || gemm_ctas < 1 || reply_ctas < 1) {
    set_error("asap_ffn_job_rows_overlap: needs a reply stream other than the job's and positive CTA counts");
    return ASAP_EINVAL;
  }
  return ffn_job_impl(experts_handle, ws_handle, R, rows, swiglu_limit, status, timeout_ns, (cudaStream_t)stream,
                      (cudaStream_t)reply_stream, gemm_ctas, reply_ctas);
}

int asap_ffn_enable_timing(uint64_t ws_handle, int32_t enable) {
  WsHandle* w = get_ws(ws_handle);
  if (!w) {
    set_error("asap_ffn_enable_timing: unknown workspace handle");
    return ASAP_EINVAL;
  }
  if (enable && !w->ev[0][0])
    for (int j = 0; j < kTimedJobs; ++j)
      for (int i = 0; i <= kTimedKernels; ++i) ASAP_CUDA(cudaEventCreate(&w->ev[j][i]));
  w->timing = enable != 0;
  w->jobs = 0;
  return ASAP_OK;
}

int asap_ffn_last_timing(uint64_t ws_handle, float* ms, int32_t n) {
  WsHandle* w = get_ws(ws_handle);
  if (!w || !ms || n < kTimedKernels || !w->ev[0][0] || w->jobs == 0) {
    set_error("asap_ffn_last_timing: timing not enabled, no job recorded, or buffer smaller than %d",
              kTimedKernels);
    return ASAP_EINVAL;
  }
  const int count = std::min(w->jobs, kTimedJobs);
  for (int i = 0; i < kTimedKernels; ++i) ms[i] = 0.f;
  for (int j = 0; j < count; ++j) {
    const int s = (w->jobs - 1 - j) % kTimedJobs;
    ASAP_CUDA(cudaEventSynchronize(w->ev[s][kTimedKernels]));
    for (int i = 0; i < kTimedKernels; ++i) {
      float t = 0.f;
      ASAP_CUDA(cudaEventElapsedTime(&t, w->ev[s][i], w->ev[s][i + 1]));
      ms[i] += t / count;
    }
  }
  return ASAP_OK;
}

int asap_ffn_job_info(uint64_t ws_handle, int32_t* n, int32_t* layer_id, uint32_t* seq, int32_t* epoch,
                      int32_t* valid, uint64_t* t_seen_ns, uint64_t* t_reply_ns, void* stream) {
  WsHandle* w = get_ws(ws_handle);
  if (!w) {
    set_error("asap_ffn_job_info: unknown workspace handle");
    return ASAP_EINVAL;
  }
  JobDesc d;
  ASAP_CUDA(cudaMemcpyAsync(&d, w->base + w->L.desc, sizeof(d), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  ASAP_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  if (n) *n = d.n;
  if (layer_id) *layer_id = d.layer;
  if (seq) *seq = d.seq;
  if (epoch) *epoch = d.epoch;
  if (valid) *valid = d.valid;
  if (t_seen_ns) *t_seen_ns = d.t_seen;
  if (t_reply_ns) *t_reply_ns = d.t_reply;
  return ASAP_OK;
}

int asap_ffn_debug_ptrs(uint64_t ws_handle, uint64_t* expert_counts, uint64_t* pair_pos, uint64_t* xq,
                        uint64_t* xq_sf, uint64_t* hq, uint64_t* hq_sf, uint64_t* y2) {
  WsHandle* w = get_ws(ws_handle);
  if (!w) {
    set_error("asap_ffn_debug_ptrs: unknown workspace handle");
    return ASAP_EINVAL;
  }
  const uint64_t b = (uint64_t)w->base;
  if (expert_counts) *expert_counts = b + w->L.ecnt;
  if (pair_pos) *pair_pos = b + w->L.pair_pos;
  if (xq) *xq = b + w->L.xq;
  if (xq_sf) *xq_sf = b + w->L.xq_sf;
  if (hq) *hq = b + w->L.hq;
  if (hq_sf) *hq_sf = b + w->L.hq_sf;
  if (y2) *y2 = b + w->L.y2;
  return ASAP_OK;
}

}  // extern "C"
