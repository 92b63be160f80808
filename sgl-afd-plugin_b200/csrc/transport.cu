// libasap transport: context/memory entry points, A-side dispatch (route + pack + doorbell) and combine.
//
// Reference behaviour replaced here (python/sgl_asap_plugin/transport/):
//   channel.py:317-362  AttnChannel.send   -> asap_dispatch (K1 route, K2 pack + doorbell release)
//   channel.py:364-377  AttnChannel.wait   -> asap_combine prologue (bounded device spin on done flags)
//   srt/layers/moe/token_dispatcher/asap.py:174-184 AsapBuffer.recv -> asap_combine body (fp32 sum -> bf16)
//   cuda_wrapper.py / memory.py IPC + host-register calls -> asap_arena_* / asap_host_*
#include <stdarg.h>
#include <string.h>

#include <errno.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"

namespace asap {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_fail(cudaError_t err, const char* what) {
  set_error("%s failed: %d %s", what, (int)err, cudaGetErrorString(err));
  return ASAP_ECUDA;
}

static int check_geometry(const asap_geometry_t* g) {
  if (!g) {
    set_error("geometry is NULL");
    return ASAP_EINVAL;
  }
  const int32_t v[7] = {g->num_a, g->group, g->slots, g->n_max, g->hidden, g->topk, g->num_f};
  const char* names[7] = {"num_a", "group", "slots", "n_max", "hidden", "topk", "num_f"};
  for (int i = 0; i < 7; ++i)
    if (v[i] < 1) {
      set_error("invalid transport geometry: %s=%d", names[i], v[i]);
      return ASAP_EINVAL;
    }
  if (g->num_a % g->group) {
    set_error("invalid transport geometry: num_a=%d is not a multiple of group=%d", g->num_a, g->group);
    return ASAP_EINVAL;
  }
  if ((uint32_t)g->n_max > kMaxTokens) {
    set_error("invalid transport geometry: n_max=%d exceeds the %u tokens a doorbell can announce", g->n_max,
              kMaxTokens);
    return ASAP_EINVAL;
  }
  return ASAP_OK;
}

// ------------------------------------------------------------------ routing workspace layout
// [0, 256)      int32 count[ASAP_MAX_F]  (rows announced to F rank f, >= 1)
// [256, 320)    int32 pad[ASAP_MAX_F]    (1 when f received no token and gets one row of ids -1)
// [320, 384)    uint32 chunks[ASAP_MAX_F]: 8-row chunks of F rank f the pack kernel has stored so far
// [384, 392)    uint64 globaltimer (ns) when the last doorbell was released
// [392, 400)    uint64 globaltimer (ns) when the combine's wait saw every done flag
// [400, 404)    uint32 doorbells released so far by the pack kernel
// [404, 512)    reserved
// [512, ...)    int32 row_of[num_f][n_max]: compacted row of token t in f's region, -1 if not routed
//               int32 tok_of[num_f][n_max]: token of compacted row r of f's region (rows < count[f])
constexpr uint64_t kWsCount = 0, kWsPad = 256, kWsSync = 320, kWsRing = 384, kWsRung = 400, kWsRows = 512;

// K1: one CTA. Backpressure wait, then the per-F-rank compacted row index of every token (ascending token
// order, a stable compaction).
constexpr int kRouteThreads = 1024;

struct Bounds {
  int32_t v[ASAP_MAX_F + 1];
};

__global__ void __launch_bounds__(kRouteThreads) dispatch_route_kernel(
    asap_geometry_t g, int32_t slot, uint32_t seq, const void* __restrict__ ids, int32_t ids_is_int64, int32_t n,
    const __grid_constant__ Bounds bounds_g, const uint8_t* result, uint8_t* ws, int32_t backpressure,
    uint64_t status, uint64_t timeout_ns) {
  __shared__ int32_t bounds[ASAP_MAX_F + 1];
  __shared__ int32_t abort_flag;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int F = g.num_f;
  if (tid <= F) bounds[tid] = bounds_g.v[tid];
  if (tid == 0) abort_flag = 0;
  __syncthreads();

  int32_t* count = reinterpret_cast<int32_t*>(ws + kWsCount);
  int32_t* pad = reinterpret_cast<int32_t*>(ws + kWsPad);
  int32_t* row_of = reinterpret_cast<int32_t*>(ws + kWsRows);
  int32_t* tok_of = row_of + (int64_t)F * g.n_max;

  // Backpressure (channel.py:337-339): the previous message of this slot must be answered by every F.
  if (backpressure && tid < F) {
    const uint32_t* done = reinterpret_cast<const uint32_t*>(result + done_off(g, tid, slot));
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    while ((int32_t)(ld_acquire_sys_u32(done) - (seq - 1u)) < 0) {
      if (globaltimer_ns() > deadline) {
        report(status, status_word(ASAP_ST_BACKPRESSURE_TIMEOUT, tid, slot, seq));
        atomicExch(&abort_flag, 1);
        break;
      }
      __nanosleep(256);
    }
  }
  __syncthreads();
  if (abort_flag) {
    if (tid < F) count[tid] = -1;  // pack sees -1 and sends nothing
    return;
  }

  // Rounds of 1024 consecutive tokens (thread i takes token base + i, so the id loads and the row-index stores
  // of a warp are contiguous): per-F-rank warp ballots, a scan over the 32 warps, a running total per F rank.
  __shared__ int32_t wcnt[32][ASAP_MAX_F];
  __shared__ int32_t run[ASAP_MAX_F];
  if (tid < ASAP_MAX_F) run[tid] = 0;
  __syncthreads();
  const uint32_t lt = (1u << lane) - 1u;
  const int64_t e_lo = bounds[0], e_end = bounds[F];
  for (int base = 0; base < n; base += kRouteThreads) {
    const int t = base + tid;
    uint32_t mask = 0;
    if (t < n) {
      for (int j = 0; j < g.topk; ++j) {
        const int64_t e = ids_is_int64 ? reinterpret_cast<const int64_t*>(ids)[(int64_t)t * g.topk + j]
                                       : reinterpret_cast<const int32_t*>(ids)[(int64_t)t * g.topk + j];
        if (e < e_lo || e >= e_end) continue;
        int f = 0;
        while (f + 1 < F && e >= bounds[f + 1]) ++f;
        mask |= 1u << f;
      }
    }
    uint32_t bal[ASAP_MAX_F];
#pragma unroll
    for (int f = 0; f < ASAP_MAX_F; ++f) {
      bal[f] = __ballot_sync(0xffffffffu, (mask >> f) & 1u);
      if (lane == 0) wcnt[warp][f] = __popc(bal[f]);
    }
    __syncthreads();
    if (warp == 0) {
      for (int f = 0; f < F; ++f) {
        const int32_t c = wcnt[lane][f];
        int32_t v = c;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int32_t u = __shfl_up_sync(0xffffffffu, v, d);
          if (lane >= d) v += u;
        }
        wcnt[lane][f] = run[f] + v - c;  // exclusive, plus the rows of earlier rounds
        __syncwarp();
        if (lane == 31) run[f] += v;
        __syncwarp();
      }
    }
    __syncthreads();
    if (t < n) {
#pragma unroll
      for (int f = 0; f < ASAP_MAX_F; ++f) {
        if (f >= F) break;
        const int32_t r = ((mask >> f) & 1u) ? wcnt[warp][f] + __popc(bal[f] & lt) : -1;
        row_of[(int64_t)f * g.n_max + t] = r;
        if (r >= 0) tok_of[(int64_t)f * g.n_max + r] = t;
      }
    }
    __syncthreads();
  }
  if (tid < F) {
    const int32_t total = run[tid];
    count[tid] = total > 0 ? total : 1;
    pad[tid] = total > 0 ? 0 : 1;
  }
  if (tid < ASAP_MAX_F) reinterpret_cast<uint32_t*>(ws + kWsSync)[tid] = 0;
  if (tid == 0) *reinterpret_cast<uint32_t*>(ws + kWsRung) = 0;
}

// K2: pack the routed rows into the F ranks' arenas and ring each F rank's doorbell as soon as all of its rows
// are stored.  The work is F ranks' compacted row lists (tok_of) cut into chunks of 8 rows, taken in phase order:
// F rank first_f first, then first_f + 1, ... (mod num_f).  A ranks start at different F ranks (first_f =
// a * num_f / num_a), so during the first phase every F rank receives one A rank's rows instead of a share of
// all of them, and its first message is complete (and its expert chain can start) after about 1 / num_f of the
// transfer.  One warp per chunk: 16-byte loads of the bf16 row, eight in flight per lane, 16-byte stores into the
// (peer) region, the row's ids and weights beside it.  After a chunk the warp's stores are fenced system-wide
// and counted; the chunk that completes an F rank releases its doorbell.
constexpr int kPackRows = 4;

struct PackArgs {
  asap_geometry_t g;
  int32_t a, slot, layer_id, n;
  uint32_t seq;
  int32_t ids_is_int64, w_is_bf16;
  int32_t first_f;
  const uint8_t* x;
  const void* ids;
  const void* w;
  uint8_t* ws;
  uint8_t* recv[ASAP_MAX_F];
  uint64_t* bell[ASAP_MAX_F];
  uint32_t epoch[ASAP_MAX_F];
};

__device__ __forceinline__ void ring_doorbell(const PackArgs& p, int f, uint32_t count) {
  __threadfence_system();
  st_release_sys_u64(reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(p.bell[f]) + bell_off(p.g, p.a, p.slot)),
                     pack_doorbell(p.seq, count, (uint32_t)p.layer_id, p.epoch[f]));
  // the last doorbell of this message records the release time (asap_dispatch_info)
  if (atomicAdd(reinterpret_cast<uint32_t*>(p.ws + kWsRung), 1u) == (uint32_t)p.g.num_f - 1u)
    *reinterpret_cast<uint64_t*>(p.ws + kWsRing) = globaltimer_ns();
}

__global__ void __launch_bounds__(256) dispatch_pack_kernel(const __grid_constant__ PackArgs p) {
  const asap_geometry_t& g = p.g;
  const int F = g.num_f;
  const int32_t* count = reinterpret_cast<const int32_t*>(p.ws + kWsCount);
  const int32_t* pad = reinterpret_cast<const int32_t*>(p.ws + kWsPad);
  const int32_t* tok_of = reinterpret_cast<const int32_t*>(p.ws + kWsRows) + (int64_t)F * g.n_max;
  uint32_t* chunks_done = reinterpret_cast<uint32_t*>(p.ws + kWsSync);
  if (count[0] < 0) return;  // backpressure timed out: send nothing
  const Offsets o = offsets_of(g);
  const int lane = threadIdx.x & 31;
  const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const uint64_t row_bytes = (uint64_t)g.hidden * 2;
  const int nvec = (int)(row_bytes / 16);
  const uint64_t roff = region_off(g, o, p.a, p.slot);

  // chunk prefix in phase order
  __shared__ int32_t first[ASAP_MAX_F + 1];
  if (threadIdx.x == 0) {
    first[0] = 0;
    for (int i = 0; i < F; ++i) {
      const int f = (p.first_f + i) % F;
      first[i + 1] = first[i] + (pad[f] ? 0 : (count[f] + kPackRows - 1) / kPackRows);
    }
  }
  __syncthreads();
  const int32_t total = first[F];

  // F ranks that got no token: one row whose ids name no expert (F's experts skip it, the reply row is 0), and
  // the doorbell at once
  if (gwarp == 0) {
    for (int f = 0; f < F; ++f) {
      if (!pad[f]) continue;
      uint8_t* base = p.recv[f] + roff;
      if (lane < g.topk) {
        reinterpret_cast<int32_t*>(base + o.ids_off)[lane] = -1;
        reinterpret_cast<float*>(base + o.w_off)[lane] = 0.f;
      }
      __syncwarp();
      if (lane == 0) ring_doorbell(p, f, 1u);
    }
  }

  for (int64_t c = gwarp; c < total; c += nwarps) {
    int i = 0;
    while (c >= first[i + 1]) ++i;
    const int f = (p.first_f + i) % F;
    const int32_t r0 = (int32_t)(c - first[i]) * kPackRows;
    const int32_t r1 = min(r0 + kPackRows, count[f]);
    uint8_t* base = p.recv[f] + roff;
    for (int32_t r = r0; r < r1; ++r) {
      const int64_t t = tok_of[(int64_t)f * g.n_max + r];
      const uint4* src = reinterpret_cast<const uint4*>(p.x + (uint64_t)t * row_bytes);
      uint4* dst = reinterpret_cast<uint4*>(base + (uint64_t)r * row_bytes);
      for (int v0 = lane; v0 < nvec; v0 += 256) {  // eight 16-byte loads in flight per lane, then their stores
        uint4 buf[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (v0 + 32 * u < nvec) buf[u] = __ldg(src + v0 + 32 * u);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (v0 + 32 * u < nvec) dst[v0 + 32 * u] = buf[u];
      }
      if (lane < g.topk) {
        const int64_t k = t * g.topk + lane;
        const int32_t id = p.ids_is_int64 ? (int32_t)reinterpret_cast<const int64_t*>(p.ids)[k]
                                          : reinterpret_cast<const int32_t*>(p.ids)[k];
        const float wt = p.w_is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.w)[k])
                                     : reinterpret_cast<const float*>(p.w)[k];
        reinterpret_cast<int32_t*>(base + o.ids_off)[(uint64_t)r * g.topk + lane] = id;
        reinterpret_cast<float*>(base + o.w_off)[(uint64_t)r * g.topk + lane] = wt;
      }
    }
    // the chunk's stores are visible system-wide before it is counted (channel.py:350 ordering: payload, then
    // doorbell); the chunk that completes F rank f rings f's doorbell
    __syncwarp();
    if (lane == 0) {
      __threadfence_system();
      const uint32_t done = atomicAdd(&chunks_done[f], 1u) + 1u;
      if (done == (uint32_t)(first[i + 1] - first[i])) ring_doorbell(p, f, (uint32_t)count[f]);
    }
  }
}

// K6: combine.  The bounded wait for the done flags runs first in its own 1-CTA kernel (wait_replies_kernel),
// so a slow F rank parks one warp, not the whole GPU; this kernel then sums the partial rows.
struct CombineArgs {
  asap_geometry_t g;
  int32_t slot, n;
  uint32_t seq;
  const uint8_t* result;
  const uint8_t* ws;
  const __nv_bfloat16* shared;
  __nv_bfloat16* out;
  uint64_t status, timeout_ns;
};

__global__ void __launch_bounds__(256, 2) combine_kernel(const __grid_constant__ CombineArgs p) {
  const asap_geometry_t& g = p.g;
  const int F = g.num_f;
  const Offsets o = offsets_of(g);
  const int32_t* row_of = reinterpret_cast<const int32_t*>(p.ws + kWsRows);
  const int lane = threadIdx.x & 31;
  const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int H = g.hidden;
  const int nvec = H / 8;  // 8 bf16 per 16-byte vector
  constexpr int U = 4;  // 16-byte vectors per lane per pass: every load of a pass is issued before its first use
  for (int64_t t = gwarp; t < p.n; t += nwarps) {
    int32_t rows[ASAP_MAX_F];
    for (int f = 0; f < F; ++f) rows[f] = row_of[(int64_t)f * g.n_max + t];
    for (int c0 = lane; c0 < nvec; c0 += 32 * U) {
      uint4 sv[U];
      if (p.shared) {
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (c0 + 32 * u < nvec)
            sv[u] = *reinterpret_cast<const uint4*>(p.shared + (uint64_t)t * H + (uint64_t)(c0 + 32 * u) * 8);
      }
      float acc[U][8];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
      for (int f = 0; f < F; ++f) {  // fp32 sum over F ranks in rank order
        if (rows[f] < 0) continue;
        const uint8_t* src = p.result + seg_off(g, o, f, p.slot) + (uint64_t)rows[f] * H * 2;
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (c0 + 32 * u < nvec) v[u] = *reinterpret_cast<const uint4*>(src + (uint64_t)(c0 + 32 * u) * 16);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (c0 + 32 * u >= nvec) continue;
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 ff = __bfloat1622float2(h[i]);
            acc[u][2 * i] += ff.x;
            acc[u][2 * i + 1] += ff.y;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c >= nvec) continue;
        uint4 r;
        __nv_bfloat162* rh = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) rh[i] = __floats2bfloat162_rn(acc[u][2 * i], acc[u][2 * i + 1]);
        if (p.shared) {  // the shared expert is added to the bf16 sum, rounded again (two roundings)
          const __nv_bfloat162* sh = reinterpret_cast<const __nv_bfloat162*>(&sv[u]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 a = __bfloat1622float2(rh[i]);
            const float2 b = __bfloat1622float2(sh[i]);
            rh[i] = __floats2bfloat162_rn(a.x + b.x, a.y + b.y);
          }
        }
        *reinterpret_cast<uint4*>(p.out + (uint64_t)t * H + (uint64_t)c * 8) = r;
      }
    }
  }
}

__global__ void wait_replies_kernel(asap_geometry_t g, int32_t slot, uint32_t seq, const uint8_t* result,
                                    uint64_t status, uint64_t timeout_ns, uint64_t* t_seen) {
  if (threadIdx.x < g.num_f) {
    const uint32_t* done = reinterpret_cast<const uint32_t*>(result + done_off(g, threadIdx.x, slot));
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    while ((int32_t)(ld_acquire_sys_u32(done) - seq) < 0) {
      if (globaltimer_ns() > deadline) {
        report(status, status_word(ASAP_ST_REPLY_TIMEOUT, threadIdx.x, slot, seq));
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
  if (threadIdx.x == 0 && t_seen) *t_seen = globaltimer_ns();
}

__global__ void write32_kernel(uint32_t* p, uint32_t v) {
  __threadfence_system();
  st_release_sys_u32(p, v);
}

__global__ void memset32_kernel(uint32_t* p, uint32_t v, uint64_t count) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cached[dev] = v;
  }
  return cached[dev];
}

// ------------------------------------------------------------------ allocation-free dispatch scratch
// Routing tables of asap_dispatch_noalloc: one per slot, in a file-scope device array that every GPU loading
// the library holds until the process exits (8 slots x (512 B + 1 MiB), about 8 MiB).
constexpr int kNoAllocSlots = 8;
constexpr uint64_t kNoAllocEntries = 1ull << 17;  // num_f * n_max routing-table rows per slot
constexpr uint64_t kNoAllocSlotBytes = kWsRows + 8ull * kNoAllocEntries;
static __device__ __align__(256) uint8_t g_noalloc_route[kNoAllocSlots][kNoAllocSlotBytes];

// Device address of g_noalloc_route on the current device, looked up once per device (the host-side symbol is
// only a stand-in and must never reach a kernel).
static int noalloc_base(uint64_t* base) {
  static std::mutex mu;
  static uint64_t cached[64] = {0};
  int dev = 0;
  ASAP_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("asap_dispatch_noalloc: device ordinal %d out of range", dev);
    return ASAP_EINVAL;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!cached[dev]) {
    void* p = nullptr;
    ASAP_CUDA(cudaGetSymbolAddress(&p, g_noalloc_route));
    cached[dev] = (uint64_t)p;
  }
  *base = cached[dev];
  return ASAP_OK;
}

}  // namespace asap

using namespace asap;

extern "C" {

const char* asap_last_error_string(void) { return g_err; }

const char* asap_version(void) { return "libasap 0.1 sm_100a"; }

int asap_geometry_offsets(const asap_geometry_t* g, asap_offsets_t* out) {
  int rc = check_geometry(g);
  if (rc) return rc;
  if (!out) {
    set_error("out is NULL");
    return ASAP_EINVAL;
  }
  const Offsets o = offsets_of(*g);
  out->ids_off = o.ids_off;
  out->w_off = o.w_off;
  out->region_bytes = o.region_bytes;
  out->recv_bytes = o.recv_bytes;
  out->host_bytes = o.host_bytes;
  out->flags_bytes = o.flags_bytes;
  out->seg_bytes = o.seg_bytes;
  out->result_bytes = o.result_bytes;
  return ASAP_OK;
}

int asap_pack_doorbell(uint32_t seq, uint32_t n_tokens, uint32_t layer_id, uint32_t epoch, uint64_t* word) {
  if (!(1 <= n_tokens && n_tokens <= kMaxTokens && layer_id <= kMaxLayer && 1 <= epoch && epoch <= kMaxEpoch)) {
    set_error("doorbell field out of range: n_tokens=%u layer_id=%u epoch=%u", n_tokens, layer_id, epoch);
    return ASAP_EINVAL;
  }
  *word = pack_doorbell(seq, n_tokens, layer_id, epoch);
  return ASAP_OK;
}

void asap_unpack_doorbell(uint64_t word, uint32_t* seq, uint32_t* n_tokens, uint32_t* layer_id, uint32_t* epoch) {
  if (seq) *seq = (uint32_t)(word & 0xffffffffull);
  if (n_tokens) *n_tokens = (uint32_t)((word >> 32) & kMaxTokens);
  if (layer_id) *layer_id = (uint32_t)((word >> 49) & kMaxLayer);
  if (epoch) *epoch = (uint32_t)(word >> 59);
}

int asap_init(int device) {
  ASAP_CUDA(cudaSetDevice(device));
  ASAP_CUDA(cudaFree(0));  // create / bind the primary context
  return ASAP_OK;
}

// What this library handed out, for asap_release: device arenas (asap_arena_alloc), peers' arenas mapped here
// (asap_arena_open) and host pages (asap_host_page_create / _open, keyed by their CPU address).
enum OwnedKind { kOwnedArena = 0, kOwnedIpc = 1, kOwnedHostPage = 2 };
struct OwnedRec {
  OwnedKind kind;
  uint64_t bytes;
  std::string unlink_path;  // host pages this process created: removed on release
};
static std::mutex g_owned_mu;
static std::unordered_map<uint64_t, OwnedRec>& owned() {
  static std::unordered_map<uint64_t, OwnedRec> m;
  return m;
}
static void own(uint64_t ptr, OwnedKind kind, uint64_t bytes = 0, const char* unlink_path = nullptr) {
  std::lock_guard<std::mutex> lk(g_owned_mu);
  owned()[ptr] = OwnedRec{kind, bytes, unlink_path ? unlink_path : ""};
}
static void disown(uint64_t ptr) {
  std::lock_guard<std::mutex> lk(g_owned_mu);
  owned().erase(ptr);
}

// Map a shared-memory file of `bytes` (created zeroed, or opened) and register it for device access.  On any
// failure everything done so far is undone (a file this call created is removed).
static int host_page_map(const char* what, const char* path, uint64_t bytes, bool create, uint64_t* host_ptr,
                         uint64_t* dev_ptr) {
  if (!path || !*path || !bytes || !host_ptr || !dev_ptr) {
    set_error("%s: need a path, bytes > 0 and non-NULL outputs", what);
    return ASAP_EINVAL;
  }
  const int fd = create ? open(path, O_RDWR | O_CREAT | O_EXCL, 0600) : open(path, O_RDWR);
  if (fd < 0) {
    set_error("%s: cannot %s %s: %s", what, create ? "create" : "open", path, strerror(errno));
    return ASAP_EINVAL;
  }
  struct stat st;
  if ((create && ftruncate(fd, (off_t)bytes) != 0) || fstat(fd, &st) != 0 || (uint64_t)st.st_size < bytes) {
    set_error("%s: %s is not %llu bytes long", what, path, (unsigned long long)bytes);
    close(fd);
    if (create) unlink(path);
    return ASAP_EINVAL;
  }
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    set_error("%s: mmap of %s failed: %s", what, path, strerror(errno));
    if (create) unlink(path);
    return ASAP_EINVAL;
  }
  uint64_t d = 0;
  const int rc = asap_host_register((uint64_t)p, bytes, &d);
  if (rc != ASAP_OK) {
    munmap(p, bytes);
    if (create) unlink(path);
    return rc;
  }
  *host_ptr = (uint64_t)p;
  *dev_ptr = d;
  own((uint64_t)p, kOwnedHostPage, bytes, create ? path : nullptr);
  return ASAP_OK;
}

int asap_host_page_create(const char* path, uint64_t bytes, uint64_t* host_ptr, uint64_t* dev_ptr) {
  return host_page_map("asap_host_page_create", path, bytes, true, host_ptr, dev_ptr);
}

int asap_host_page_open(const char* path, uint64_t bytes, uint64_t* host_ptr, uint64_t* dev_ptr) {
  return host_page_map("asap_host_page_open", path, bytes, false, host_ptr, dev_ptr);
}

int asap_release(uint64_t ptr) {
  OwnedRec rec;
  {
    std::lock_guard<std::mutex> lk(g_owned_mu);
    auto it = owned().find(ptr);
    if (it == owned().end()) {
      set_error("asap_release: 0x%llx was not handed out by this library (or is already released)",
                (unsigned long long)ptr);
      return ASAP_EINVAL;
    }
    rec = it->second;
    owned().erase(it);
  }
  switch (rec.kind) {
    case kOwnedArena:
      ASAP_CUDA(cudaFree((void*)ptr));
      return ASAP_OK;
    case kOwnedIpc:
      ASAP_CUDA(cudaIpcCloseMemHandle((void*)ptr));
      return ASAP_OK;
    case kOwnedHostPage: {
      const cudaError_t err = cudaHostUnregister((void*)ptr);
      munmap((void*)ptr, rec.bytes);
      if (!rec.unlink_path.empty()) unlink(rec.unlink_path.c_str());
      return err == cudaSuccess ? ASAP_OK : cuda_fail(err, "cudaHostUnregister");
    }
  }
  return ASAP_EINVAL;
}

int asap_arena_alloc(uint64_t bytes, uint64_t* dev_ptr, uint8_t ipc_handle[64]) {
  if (!bytes || !dev_ptr) {
    set_error("asap_arena_alloc: bytes must be > 0 and dev_ptr non-NULL");
    return ASAP_EINVAL;
  }
  void* p = nullptr;
  ASAP_CUDA(cudaMalloc(&p, bytes));
  if (ipc_handle) {
    cudaIpcMemHandle_t h;
    cudaError_t err = cudaIpcGetMemHandle(&h, p);
    if (err != cudaSuccess) {
      cudaFree(p);
      return cuda_fail(err, "cudaIpcGetMemHandle");
    }
    memcpy(ipc_handle, &h, 64);
  }
  *dev_ptr = (uint64_t)p;
  own(*dev_ptr, kOwnedArena);
  return ASAP_OK;
}

int asap_arena_free(uint64_t dev_ptr) {
  disown(dev_ptr);
  ASAP_CUDA(cudaFree((void*)dev_ptr));
  return ASAP_OK;
}

int asap_arena_open(const uint8_t ipc_handle[64], uint64_t* dev_ptr) {
  if (!ipc_handle || !dev_ptr) {
    set_error("asap_arena_open: NULL argument");
    return ASAP_EINVAL;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, 64);
  void* p = nullptr;
  ASAP_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *dev_ptr = (uint64_t)p;
  own(*dev_ptr, kOwnedIpc);
  return ASAP_OK;
}

int asap_arena_close(uint64_t dev_ptr) {
  disown(dev_ptr);
  ASAP_CUDA(cudaIpcCloseMemHandle((void*)dev_ptr));
  return ASAP_OK;
}

int asap_host_register(uint64_t host_ptr, uint64_t bytes, uint64_t* dev_ptr) {
  if (!host_ptr || !bytes || !dev_ptr) {
    set_error("asap_host_register: NULL pointer or zero size");
    return ASAP_EINVAL;
  }
  ASAP_CUDA(cudaHostRegister((void*)host_ptr, bytes, cudaHostRegisterPortable | cudaHostRegisterMapped));
  void* d = nullptr;
  cudaError_t err = cudaHostGetDevicePointer(&d, (void*)host_ptr, 0);
  if (err != cudaSuccess) {
    cudaHostUnregister((void*)host_ptr);
    return cuda_fail(err, "cudaHostGetDevicePointer");
  }
  *dev_ptr = (uint64_t)d;
  return ASAP_OK;
}

int asap_host_unregister(uint64_t host_ptr) {
  ASAP_CUDA(cudaHostUnregister((void*)host_ptr));
  return ASAP_OK;
}

int asap_memset32(uint64_t dev_ptr, uint32_t value, uint64_t count, void* stream) {
  if (!count) return ASAP_OK;
  const int blocks = (int)std::min<uint64_t>((count + 255) / 256, 4096);
  memset32_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((uint32_t*)dev_ptr, value, count);
  ASAP_CHECK_LAUNCH("memset32_kernel");
  return ASAP_OK;
}

int asap_write32(uint64_t dev_ptr, uint32_t value, void* stream) {
  write32_kernel<<<1, 1, 0, (cudaStream_t)stream>>>((uint32_t*)dev_ptr, value);
  ASAP_CHECK_LAUNCH("write32_kernel");
  return ASAP_OK;
}

uint64_t asap_route_ws_bytes(const asap_geometry_t* g) {
  if (!g || g->num_f < 1 || g->n_max < 1) return 0;
  return kWsRows + (uint64_t)g->num_f * g->n_max * 8;  // row_of and tok_of
}

static int dispatch_impl(const asap_geometry_t* g, int32_t a, int32_t slot, uint32_t seq, int32_t layer_id,
                         const int32_t* epochs, uint64_t x, uint64_t ids, int32_t ids_is_int64, uint64_t w,
                         int32_t w_is_bf16, int32_t n, const int32_t* expert_bounds, const uint64_t* recv,
                         const uint64_t* bells, uint64_t result, uint64_t route_ws, int32_t backpressure,
                         uint64_t status, uint64_t timeout_ns, void* stream) {
  int rc = check_geometry(g);
  if (rc) return rc;
  if (g->num_f > ASAP_MAX_F || g->topk > 32) {
    set_error("asap_dispatch: num_f=%d (max %d) / topk=%d (max 32) unsupported", g->num_f, ASAP_MAX_F, g->topk);
    return ASAP_EINVAL;
  }
  if (a < 0 || a >= g->num_a || slot < 0 || slot >= g->slots || n < 1 || n > g->n_max) {
    set_error("slot %d / n_tokens %d / A rank %d outside the geometry", slot, n, a);
    return ASAP_EINVAL;
  }
  if ((uint32_t)layer_id > kMaxLayer) {
    set_error("doorbell field out of range: layer_id=%d", layer_id);
    return ASAP_EINVAL;
  }
  if (g->hidden % 8) {
    set_error("asap_dispatch: hidden=%d must be a multiple of 8", g->hidden);
    return ASAP_EINVAL;
  }
  if (!x || !ids || !w || !result || !route_ws || !recv || !bells || !epochs || !expert_bounds) {
    set_error("asap_dispatch: NULL pointer argument");
    return ASAP_EINVAL;
  }
  if ((x & 15) || (route_ws & 15)) {
    set_error("asap_dispatch: x and route_ws must be 16-byte aligned");
    return ASAP_EINVAL;
  }
  for (int f = 0; f < g->num_f; ++f) {
    if (epochs[f] < 1 || (uint32_t)epochs[f] > kMaxEpoch) {
      set_error("doorbell field out of range: epoch=%d (F rank %d)", epochs[f], f);
      return ASAP_EINVAL;
    }
    if (expert_bounds[f + 1] < expert_bounds[f]) {
      set_error("asap_dispatch: expert_bounds must be non-decreasing");
      return ASAP_EINVAL;
    }
  }
  cudaStream_t st = (cudaStream_t)stream;
  Bounds bounds;
  memset(&bounds, 0, sizeof(bounds));
  for (int f = 0; f <= g->num_f; ++f) bounds.v[f] = expert_bounds[f];
  dispatch_route_kernel<<<1, kRouteThreads, 0, st>>>(*g, slot, seq, (const void*)ids, ids_is_int64, n, bounds,
                                                     (const uint8_t*)result, (uint8_t*)route_ws, backpressure,
                                                     status, timeout_ns);
  ASAP_CHECK_LAUNCH("dispatch_route_kernel");
  PackArgs p;
  memset(&p, 0, sizeof(p));
  p.g = *g;
  p.a = a;
  p.slot = slot;
  p.layer_id = layer_id;
  p.n = n;
  p.seq = seq;
  p.ids_is_int64 = ids_is_int64;
  p.w_is_bf16 = w_is_bf16;
  p.x = (const uint8_t*)x;
  p.ids = (const void*)ids;
  p.w = (const void*)w;
  p.ws = (uint8_t*)route_ws;
  p.first_f = (int32_t)((int64_t)a * g->num_f / g->num_a);
  for (int f = 0; f < g->num_f; ++f) {
    p.recv[f] = (uint8_t*)recv[f];
    p.bell[f] = (uint64_t*)bells[f];
    p.epoch[f] = (uint32_t)epochs[f];
  }
  // one warp per 4-row chunk: at most num_f * n / 4 + num_f chunks, and at most 4 CTAs of 8 warps per SM
  const int warps = 8;
  const int64_t chunks = ((int64_t)g->num_f * n + kPackRows - 1) / kPackRows + g->num_f;
  const int blocks = (int)std::min<int64_t>((chunks + warps - 1) / warps, (int64_t)sm_count() * 4);
  dispatch_pack_kernel<<<blocks, warps * 32, 0, st>>>(p);
  ASAP_CHECK_LAUNCH("dispatch_pack_kernel");
  return ASAP_OK;
}

int asap_dispatch(const asap_geometry_t* g, int32_t a, int32_t slot, uint32_t seq, int32_t layer_id,
                  const int32_t* epochs, uint64_t x, uint64_t ids, int32_t ids_is_int64, uint64_t w,
                  int32_t w_is_bf16, int32_t n, const int32_t* expert_bounds, const uint64_t* recv,
                  const uint64_t* bells, uint64_t result, uint64_t route_ws, int32_t backpressure,
                  uint64_t status, uint64_t timeout_ns, void* stream) {
  return dispatch_impl(g, a, slot, seq, layer_id, epochs, x, ids, ids_is_int64, w, w_is_bf16, n, expert_bounds, recv,
                       bells, result, route_ws, backpressure, status, timeout_ns, stream);
}

int asap_combine(const asap_geometry_t* g, int32_t slot, uint32_t seq, int32_t n, uint64_t result,
                 uint64_t route_ws, uint64_t shared, uint64_t out, uint64_t status, uint64_t timeout_ns,
                 void* stream) {
  int rc = check_geometry(g);
  if (rc) return rc;
  if (g->num_f > ASAP_MAX_F || slot < 0 || slot >= g->slots || n < 1 || n > g->n_max) {
    set_error("asap_combine: slot %d / n_tokens %d outside the geometry", slot, n);
    return ASAP_EINVAL;
  }
  if (g->hidden % 8 || !result || !route_ws || !out || (out & 15) || (shared & 15)) {
    set_error("asap_combine: hidden must be a multiple of 8 and out/shared 16-byte aligned, non-NULL");
    return ASAP_EINVAL;
  }
  CombineArgs p;
  p.g = *g;
  p.slot = slot;
  p.n = n;
  p.seq = seq;
  p.result = (const uint8_t*)result;
  p.ws = (const uint8_t*)route_ws;
  p.shared = (const __nv_bfloat16*)shared;
  p.out = (__nv_bfloat16*)out;
  p.status = status;
  p.timeout_ns = timeout_ns;
  wait_replies_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(*g, slot, seq, (const uint8_t*)result, status, timeout_ns,
                                                          reinterpret_cast<uint64_t*>(route_ws + kWsRing + 8));
  ASAP_CHECK_LAUNCH("wait_replies_kernel");
  const int warps = 8;  // one token per warp; two CTAs of 8 warps per SM, one wave
  int blocks = std::min((n + warps - 1) / warps, sm_count() * 2);
  combine_kernel<<<blocks, warps * 32, 0, (cudaStream_t)stream>>>(p);
  ASAP_CHECK_LAUNCH("combine_kernel");
  return ASAP_OK;
}

int asap_dispatch_info(uint64_t route_ws, int32_t num_f, int32_t* counts, uint64_t* t_ring_ns,
                       uint64_t* t_replies_ns, void* stream) {
  if (!route_ws || num_f < 1 || num_f > ASAP_MAX_F) {
    set_error("asap_dispatch_info: NULL workspace or num_f %d outside [1, %d]", num_f, ASAP_MAX_F);
    return ASAP_EINVAL;
  }
  uint8_t head[kWsRows];
  ASAP_CUDA(cudaMemcpyAsync(head, (const void*)route_ws, kWsRows, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  ASAP_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  if (counts) memcpy(counts, head + kWsCount, sizeof(int32_t) * num_f);
  if (t_ring_ns) memcpy(t_ring_ns, head + kWsRing, sizeof(uint64_t));
  if (t_replies_ns) memcpy(t_replies_ns, head + kWsRing + 8, sizeof(uint64_t));
  return ASAP_OK;
}

int asap_wait_replies(const asap_geometry_t* g, int32_t slot, uint32_t seq, uint64_t result, uint64_t status,
                      uint64_t timeout_ns, void* stream) {
  int rc = check_geometry(g);
  if (rc) return rc;
  if (g->num_f > ASAP_MAX_F || slot < 0 || slot >= g->slots || !result) {
    set_error("asap_wait_replies: slot %d outside the geometry or NULL result", slot);
    return ASAP_EINVAL;
  }
  wait_replies_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(*g, slot, seq, (const uint8_t*)result, status, timeout_ns,
                                                          nullptr);
  ASAP_CHECK_LAUNCH("wait_replies_kernel");
  return ASAP_OK;
}

// Allocation-free variant of asap_dispatch (no counterpart in the reference): the routing table lives in
// g_noalloc_route[slot] instead of a caller-allocated workspace; *route_ws_out receives its device address for
// asap_combine / asap_wait_replies.  Checks, kernels and results are those of asap_dispatch.
int asap_dispatch_noalloc(const asap_geometry_t* g, int32_t a, int32_t slot, uint32_t seq, int32_t layer_id,
                          const int32_t* epochs, uint64_t x, uint64_t ids, int32_t ids_is_int64, uint64_t w,
                          int32_t w_is_bf16, int32_t n, const int32_t* expert_bounds, const uint64_t* recv,
                          const uint64_t* bells, uint64_t result, int32_t backpressure, uint64_t status,
                          uint64_t timeout_ns, void* stream, uint64_t* route_ws_out) {
  int rc = check_geometry(g);
  if (rc) return rc;
  if (!route_ws_out) {
    set_error("asap_dispatch_noalloc: route_ws_out is NULL");
    return ASAP_EINVAL;
  }
  if (slot < 0 || slot >= kNoAllocSlots) {
    set_error("asap_dispatch_noalloc: slot %d outside the %d slots of the static routing tables", slot,
              kNoAllocSlots);
    return ASAP_EINVAL;
  }
  if ((uint64_t)g->num_f * (uint64_t)g->n_max > kNoAllocEntries) {
    set_error("asap_dispatch_noalloc: num_f * n_max = %llu exceeds the static maximum of %llu routing-table rows "
              "per slot; use asap_dispatch with a workspace of asap_route_ws_bytes()",
              (unsigned long long)g->num_f * (unsigned long long)g->n_max, (unsigned long long)kNoAllocEntries);
    return ASAP_EINVAL;
  }
  uint64_t base = 0;
  rc = noalloc_base(&base);
  if (rc) return rc;
  const uint64_t ws = base + (uint64_t)slot * kNoAllocSlotBytes;
  rc = asap_dispatch(g, a, slot, seq, layer_id, epochs, x, ids, ids_is_int64, w, w_is_bf16, n, expert_bounds,
                     recv, bells, result, ws, backpressure, status, timeout_ns, stream);
  if (rc) return rc;
  *route_ws_out = ws;
  return ASAP_OK;
}

}  // extern "C"
