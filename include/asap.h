/*
 * asap.h — C ABI of libasap, the B200 (sm_100a) data path of the A->F->A MoE round trip.
 *
 * The reference plugin (Socratesa/sgl-afd-plugin, python/sgl_asap_plugin/) moves data with CUDA driver
 * copy engines and stream memory operations bound through ctypes (transport/cuda_wrapper.py) and leaves
 * the expert math to SGLang FusedMoE / FlashInfer.  libasap replaces those driver calls and the expert
 * call with kernels that do the same work on the SMs:
 *
 *   A rank                                   F rank f
 *   asap_dispatch  (route + pack + doorbell) -> RecvArena region(a, s)   (replaces channel.py:335-355)
 *                                             asap_ffn_wait  (doorbell)   (replaces server.py:262-294 poll)
 *                                             asap_ffn_job   (experts + reply into A's ResultArena)
 *                                                                         (replaces scheduler.py:387-436 and
 *                                                                          server.py:340-350)
 *   asap_combine   (wait done flags + sum partials + shared expert)      (replaces channel.py:364-377 and
 *                                                                          token_dispatcher/asap.py:174-184)
 *
 * Conventions
 *  - Every pointer argument that names device memory is a uint64_t device address (UVA): local memory,
 *    a peer's IPC mapping, or the device alias of registered host memory.
 *  - `stream` is a cudaStream_t passed as void*. 0 means the legacy default stream.
 *  - Every function returns 0 (ASAP_OK) or a negative ASAP_E* code and never throws; the message of the
 *    last failure on the calling thread is in asap_last_error_string().
 *  - Device-side failures (a bounded wait that ran out, a doorbell that does not decode) never trap: the
 *    kernel writes an asap status word to `status` (first failure wins) and returns; the host reads it.
 *    Status word: bits 0-7 code (ASAP_ST_*), 8-15 F rank, 16-23 slot, 24-31 reserved, 32-63 seq.
 *  - The arena byte layout is the reference's transport/layout.py Geometry, byte for byte.
 */
#ifndef ASAP_H_
#define ASAP_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ASAP_OK 0
#define ASAP_EINVAL (-1)    /* bad argument (reference: ValueError) */
#define ASAP_ECUDA (-2)     /* a CUDA runtime/driver call failed */
#define ASAP_ETIMEOUT (-3)  /* a host-side bounded wait ran out */
#define ASAP_EPOISONED (-4) /* reserved for the channel state machine */

/* device status codes (low byte of the status word) */
#define ASAP_ST_OK 0
#define ASAP_ST_BACKPRESSURE_TIMEOUT 1 /* dispatch: done[f][slot] never reached seq-1 */
#define ASAP_ST_DOORBELL_TIMEOUT 2     /* ffn_wait: the doorbell never advanced */
#define ASAP_ST_BAD_DOORBELL 3         /* ffn_wait: stale epoch or n_tokens out of range */
#define ASAP_ST_REPLY_TIMEOUT 4        /* combine: done[f][slot] never reached seq */
#define ASAP_ST_PIPELINE_TIMEOUT 5     /* a GEMM pipeline barrier never completed */
#define ASAP_ST_BAD_JOB 6              /* ffn_job: the job descriptor is not valid */

#define ASAP_MAX_F 16          /* F ranks one A rank can address */
#define ASAP_MAX_LOCAL_EXPERTS 256
#define ASAP_MAX_JOB_ROWS 8 /* messages one F job may answer at once (asap_ffn_*_rows) */

/* Transport geometry: the fields of transport/layout.py:115-125 (Geometry), same meaning. */
typedef struct {
  int32_t num_a, group, slots, n_max, hidden, topk, num_f;
} asap_geometry_t;

/* Offsets of the geometry, computed exactly as transport/layout.py:142-191 does. */
typedef struct {
  uint64_t ids_off, w_off, region_bytes, recv_bytes, host_bytes, flags_bytes, seg_bytes, result_bytes;
} asap_offsets_t;

/* ---------------------------------------------------------------- context and memory ----------- */

/* The message of the last failed call on this thread ("" if none). */
const char* asap_last_error_string(void);

/* Library version string. */
const char* asap_version(void);

/* Offsets of a geometry (replaces layout.py Geometry properties); ASAP_EINVAL on an invalid geometry
 * (layout.py:127-140 rules). */
int asap_geometry_offsets(const asap_geometry_t* g, asap_offsets_t* out);

/* Pack / unpack the 64-bit doorbell (layout.py:92-112). pack returns ASAP_EINVAL on out-of-range fields. */
int asap_pack_doorbell(uint32_t seq, uint32_t n_tokens, uint32_t layer_id, uint32_t epoch, uint64_t* word);
void asap_unpack_doorbell(uint64_t word, uint32_t* seq, uint32_t* n_tokens, uint32_t* layer_id,
                          uint32_t* epoch);

/* Make `device` current for this thread (cudaSetDevice; the primary context torch also uses).
 * Replaces cuda_wrapper.py:172-183 Device.activate. */
int asap_init(int device);

/* Device memory that peers can map: cudaMalloc + cudaIpcGetMemHandle (64 handle bytes).
 * Replaces memory.py:67-74 IpcMemory.device / cuda_wrapper.py:190-214. */
int asap_arena_alloc(uint64_t bytes, uint64_t* dev_ptr, uint8_t ipc_handle[64]);
int asap_arena_free(uint64_t dev_ptr);

/* Map a peer's arena (cudaIpcOpenMemHandle, lazy peer access) / unmap it.
 * Replaces memory.py:94-96 IpcMemory.open / cuda_wrapper.py:217-226. */
int asap_arena_open(const uint8_t ipc_handle[64], uint64_t* dev_ptr);
int asap_arena_close(uint64_t dev_ptr);

/* Pin an existing host mapping (a /dev/shm doorbell page) for device access -> its device address.
 * Replaces cuda_wrapper.py:230-239 host_register / host_unregister (memory.py:98-116). */
int asap_host_register(uint64_t host_ptr, uint64_t bytes, uint64_t* dev_ptr);
int asap_host_unregister(uint64_t host_ptr);

/* A shared-memory host page (doorbell page, status words) at `path` (e.g. under /dev/shm): created zeroed (fails
 * when the file exists) or opened (fails when it is shorter than `bytes`), mapped here and registered for device
 * access -> its CPU and device addresses.  The owner creates, peers open (memory.py:87-126 does the same in
 * Python).  Released with asap_release(host_ptr). */
int asap_host_page_create(const char* path, uint64_t bytes, uint64_t* host_ptr, uint64_t* dev_ptr);
int asap_host_page_open(const char* path, uint64_t bytes, uint64_t* host_ptr, uint64_t* dev_ptr);

/* Release whatever this library handed out at `ptr`: an asap_arena_alloc arena (freed), an asap_arena_open mapping
 * (unmapped), or a host page by its CPU address (unregistered, unmapped, and its file removed when this process
 * created it) -- the Shared.release of memory.py:34-45.  ASAP_EINVAL for any other pointer, or a second release. */
int asap_release(uint64_t ptr);

/* Fill `count` 32-bit words with `value` on `stream` (replaces cuda_wrapper.py:197-202 memset32). */
int asap_memset32(uint64_t dev_ptr, uint32_t value, uint64_t count, void* stream);

/* Enqueue one release-ordered 32-bit store on `stream` (replaces cuda_wrapper.py:258-260 write32; used by
 * the watchdog to release waits). */
int asap_write32(uint64_t dev_ptr, uint32_t value, void* stream);

/* Bytes of the per-slot routing workspace asap_dispatch fills and asap_combine reads: 512 + 8 * num_f * n_max
 * (each F rank's token -> row table and its row -> token list). */
uint64_t asap_route_ws_bytes(const asap_geometry_t* g);

/* ---------------------------------------------------------------- A side ------------------------ */

/* One message of A rank `a`, slot `slot`, to every F rank (replaces channel.py:317-362 AttnChannel.send
 * and its 3 copies + doorbell per F rank).
 *  x        bf16 [n, hidden]
 *  ids      [n, topk] logical expert ids, int32 (ids_is_int64=0) or int64 (1); ids outside
 *           [0, expert_bounds[num_f]) go to no F rank
 *  w        [n, topk] top-k weights, fp32 (w_is_bf16=0) or bf16 (1)
 *  expert_bounds[num_f+1]  F rank f owns experts [expert_bounds[f], expert_bounds[f+1])
 *  recv[f]  device address of F rank f's RecvArena (mapped here)
 *  bells[f] device address of F rank f's doorbell page (mapped here)
 *  epochs[f] the epoch F rank f gave this rank at the handshake (1..31)
 *  result   this rank's ResultArena (done flags at done_off(f, slot))
 *  route_ws asap_route_ws_bytes() of device memory for this slot; combine reads it
 * Each F rank receives only the tokens routed to it (compacted, ascending token order); the doorbell
 * announces that count. A rank that receives no token gets one row whose ids are all -1.
 * Each F rank's doorbell is released as soon as its own rows are stored, and A rank a sends to F rank
 * a*num_f/num_a first, then the next ones in turn, so that concurrent A ranks start on different F ranks and
 * each F rank has a complete first message after about 1/num_f of the transfer.
 * The kernel first waits (bounded by timeout_ns) until done[f][slot] >= seq-1 for every f when
 * backpressure != 0; on timeout it writes ASAP_ST_BACKPRESSURE_TIMEOUT and sends nothing. */
int asap_dispatch(const asap_geometry_t* g, int32_t a, int32_t slot, uint32_t seq, int32_t layer_id,
                  const int32_t* epochs, uint64_t x, uint64_t ids, int32_t ids_is_int64, uint64_t w,
                  int32_t w_is_bf16, int32_t n, const int32_t* expert_bounds, const uint64_t* recv,
                  const uint64_t* bells, uint64_t result, uint64_t route_ws, int32_t backpressure,
                  uint64_t status, uint64_t timeout_ns, void* stream);

/* Wait (bounded by timeout_ns) until done[f][slot] >= seq for every f, then
 * out[t] = bf16( sum_f seg(f,slot)[row_of(f,t)] in fp32, f ascending )   [asap.py:178-184]
 * and, when shared != 0, out[t] = bf16(float(out[t]) + float(shared[t]))  [the shared-expert add].
 * out/shared: bf16 [n, hidden]. On timeout writes ASAP_ST_REPLY_TIMEOUT (out is then garbage). */
int asap_combine(const asap_geometry_t* g, int32_t slot, uint32_t seq, int32_t n, uint64_t result,
                 uint64_t route_ws, uint64_t shared, uint64_t out, uint64_t status, uint64_t timeout_ns,
                 void* stream);

/* Read back a routing workspace after a dispatch and its combine (debug/measurement): the row count announced to
 * each F rank, the globaltimer (ns) at which the last of its doorbells was released and the one at which asap_combine's wait
 * saw every done flag. Synchronizes `stream`. */
int asap_dispatch_info(uint64_t route_ws, int32_t num_f, int32_t* counts, uint64_t* t_ring_ns,
                       uint64_t* t_replies_ns, void* stream);

/* Allocation-free asap_dispatch (no counterpart in the reference).  Some callers cannot allocate device memory:
 * an attention rank whose free memory SGLang has already handed to the KV-cache pool, or a host that binds this
 * ABI from another language and only holds the transport's mapped arenas.  This entry point needs no routing
 * workspace from them: the routing table of each slot lives in a static device array inside the library (8
 * slots, num_f * n_max <= 131072 rows per slot, about 8 MiB held by every GPU that loads the library until the
 * process exits), and *route_ws_out returns its device address for asap_combine / asap_wait_replies.  Larger
 * geometries or slot >= 8 are rejected with ASAP_EINVAL.  The first call on a device looks the array up
 * (cudaGetSymbolAddress) with that device current; make that first call before any stream capture.  It calls no
 * cudaMalloc/cudaFree.  Every call shares the array: a slot's table keeps the last call's contents until the next
 * dispatch on that slot overwrites it, so dispatches on one slot that overlap on the GPU (or a dispatch that
 * overlaps the combine still reading the slot's table) race.  The 8 tables are shared by every caller on the
 * device: every A replica and geometry of the process that dispatches through this entry point on that GPU.  The
 * looked-up address is cached per device ordinal for the life of the process: do not use this entry point across a
 * cudaDeviceReset (or any reset of the device's primary context).  Otherwise identical to asap_dispatch. */
int asap_dispatch_noalloc(const asap_geometry_t* g, int32_t a, int32_t slot, uint32_t seq, int32_t layer_id,
                          const int32_t* epochs, uint64_t x, uint64_t ids, int32_t ids_is_int64, uint64_t w,
                          int32_t w_is_bf16, int32_t n, const int32_t* expert_bounds, const uint64_t* recv,
                          const uint64_t* bells, uint64_t result, int32_t backpressure, uint64_t status,
                          uint64_t timeout_ns, void* stream, uint64_t* route_ws_out);

/* Wait (bounded by timeout_ns) until done[f][slot] >= seq for every f, without reading the segments
 * (replaces channel.py:364-377 AttnChannel.wait for callers that sum the segments themselves). */
int asap_wait_replies(const asap_geometry_t* g, int32_t slot, uint32_t seq, uint64_t result, uint64_t status,
                      uint64_t timeout_ns, void* stream);

/* ---------------------------------------------------------------- F side ------------------------ */

/* Routed experts of one layer on one F rank, MXFP4 (E2M1 values, E8M0 scale per 32 along K).
 * Layouts (all device memory, written by the host-side weight packer):
 *  w13     [num_local][2*inter][hidden/2] bytes: E2M1 pairs, low nibble first. Rows are the gate (W1) and
 *          up (W3) projections interleaved in blocks of 128: rows [256b, 256b+128) = gate[128b, 128b+128),
 *          rows [256b+128, 256b+256) = up[128b, 128b+128).
 *  w13_sf  [num_local][hidden/128][2*inter/128][512] E8M0 scale atoms: one 512-byte atom per 128 rows x 4
 *          32-wide K blocks, byte (r % 32) * 16 + ((r / 32) % 4) * 4 + kb % 4 for row r, block kb
 *  w2      [num_local][hidden][inter/2] bytes
 *  w2_sf   [num_local][inter/128][hidden/128][512]
 * hidden % 256 == 0, inter % 128 == 0. */
typedef struct {
  int32_t num_local, expert_base, hidden, inter;
  uint64_t w13, w13_sf, w2, w2_sf;
} asap_mxfp4_experts_t;

/* Build the TMA descriptors of a layer's weights once; *handle names them in asap_ffn_job. */
int asap_experts_register(const asap_mxfp4_experts_t* e, uint64_t* handle);
int asap_experts_release(uint64_t handle);

/* Routed experts of one layer on one F rank, FP8 E4M3 with fp32 scales per 128 x 128 block -- the layout of
 * SGLang's block-quantised FusedMoE (w13_weight / w13_weight_scale_inv, w2_weight / w2_weight_scale_inv of a
 * DeepSeek-style FP8 checkpoint, weight = e4m3 * scale), unchanged:
 *  w13        [num_local][2*inter][hidden] E4M3: gate (W1) rows [0, inter), up (W3) rows [inter, 2*inter)
 *  w13_scale  [num_local][2*inter/128][hidden/128] fp32
 *  w2         [num_local][hidden][inter] E4M3
 *  w2_scale   [num_local][hidden/128][inter/128] fp32
 * Activations are quantised to E4M3 per 1 x 128 with an fp32 scale amax / 448 (as SGLang's per-token-group
 * FP8 quantisation).  hidden % 256 == 0, inter % 128 == 0.  The handle is used with asap_ffn_job like an MXFP4
 * one; asap_experts_release frees either kind. */
typedef struct {
  int32_t num_local, expert_base, hidden, inter;
  uint64_t w13, w13_scale, w2, w2_scale;
} asap_fp8_experts_t;

int asap_experts_register_fp8(const asap_fp8_experts_t* e, uint64_t* handle);

/* F-rank job workspace for up to n_max tokens of top-k `topk` (device memory, owned by the caller).
 * Size from asap_ffn_ws_bytes; asap_ffn_ws_register builds its TMA descriptors. */
uint64_t asap_ffn_ws_bytes(int32_t n_max, int32_t topk, int32_t num_local, int32_t hidden, int32_t inter);
int asap_ffn_ws_register(uint64_t ws, int32_t n_max, int32_t topk, int32_t num_local, int32_t hidden,
                         int32_t inter, uint64_t* handle);
int asap_ffn_ws_release(uint64_t handle);

/* Device-side doorbell wait (replaces the CPU poll of server.py:262-320 for one (a, slot)):
 * spin (bounded by timeout_ns) on the 64-bit doorbell at `bell` until its seq is cyclically ahead of
 * last_seq, decode it, check epoch == expect_epoch and 1 <= n <= n_max, and write the job descriptor
 * into the workspace. A failure writes ASAP_ST_DOORBELL_TIMEOUT / ASAP_ST_BAD_DOORBELL and an invalid
 * descriptor (asap_ffn_job then does nothing). */
int asap_ffn_wait(uint64_t ws_handle, uint64_t bell, uint32_t last_seq, int32_t expect_epoch,
                  int32_t n_max, uint64_t status, uint64_t timeout_ns, void* stream);

/* Host-side alternative to asap_ffn_wait: write a job descriptor the host decoded itself. */
int asap_ffn_post(uint64_t ws_handle, uint32_t seq, int32_t n, int32_t layer_id, int32_t epoch,
                  void* stream);

/* Joined jobs (the reference's Job with several Rows, transport/server.py:322-337 and scheduler.py:387-436, here
 * also across A replicas): one F job answers `rows` <= ASAP_MAX_JOB_ROWS messages of the same layer at once, the
 * experts' weights read once for all of them.  asap_ffn_wait_rows waits for every row's doorbell (arrays of
 * `rows` entries: doorbell address, last seq, expected epoch); asap_ffn_post_rows is its host-side form.  The
 * workspace must hold the rows' tokens together (asap_ffn_ws_bytes with n_max = the sum).  A mismatch of the rows'
 * layers or an overflow writes ASAP_ST_BAD_JOB and an invalid descriptor. */
int asap_ffn_wait_rows(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint32_t* last_seqs,
                       const int32_t* expect_epochs, int32_t n_max, uint64_t status, uint64_t timeout_ns,
                       void* stream);
int asap_ffn_post_rows(uint64_t ws_handle, int32_t rows, const uint32_t* seqs, const int32_t* ns, int32_t layer_id,
                       const int32_t* epochs, void* stream);

/* asap_ffn_wait_rows whose last consumed seq per row lives in device memory (seq_states: device addresses of
 * uint32 words, one per row): the wait reads it and stores the seq it consumed, so the same launch -- or a CUDA
 * graph captured around it -- waits for the next message each time it runs. */
int asap_ffn_wait_state(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint64_t* seq_states,
                        const int32_t* expect_epochs, int32_t n_max, uint64_t status, uint64_t timeout_ns,
                        void* stream);

/* Answer ONE message: the first ready one among `rows` doorbells, in round-robin order after the row answered last
 * (int32 device word rr_state) -- the reference's FfnServer.poll order over ready doorbells (server.py:270-275) on
 * the device.  Sequence words as in asap_ffn_wait_state.  The job descriptor then holds one row whose view is the
 * picked index: pass asap_ffn_job_rows all `rows` views (same order); it answers the picked message only. */
int asap_ffn_wait_any(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint64_t* seq_states,
                      const int32_t* expect_epochs, int32_t n_max, uint64_t rr_state, uint64_t status,
                      uint64_t timeout_ns, void* stream);

/* Answer every message of this round not answered yet: row r is left out when its sequence word (as in
 * asap_ffn_wait_state) already reached round_seqs[r] -- typically taken by an asap_ffn_wait_any job before it --
 * and every other row's next message is awaited and joined into one job (row states in row order, each row's view
 * its index: pass asap_ffn_job_rows all `rows` views).  A job with no row left is empty: not valid, no error, no
 * reply.  With the reference's one-message-at-a-time poll (server.py:262-294) an F rank serving several A replicas
 * runs one job per message; answering the first ready message alone and the rest of the round together starts as
 * early and runs the remaining messages as one larger job. */
int asap_ffn_wait_rest(uint64_t ws_handle, int32_t rows, const uint64_t* bells, const uint64_t* seq_states,
                       const uint32_t* round_seqs, const int32_t* expect_epochs, int32_t n_max, uint64_t status,
                       uint64_t timeout_ns, void* stream);

/* CUDA graphs of F chains (the analogue of the reference's FfnCudaGraphRunner, srt/model_executor/runner/
 * ffn_cuda_graph_runner.py:75-92, here with no host copy into static buffers: the chain sizes itself on the
 * device).  asap_graph_begin starts capturing `stream` (thread-local mode): the asap_* launches on it until
 * asap_graph_end are recorded, not run; asap_graph_end instantiates them (*graph names the executable graph);
 * asap_graph_launch replays it on a stream; asap_graph_release frees it. */
int asap_graph_begin(void* stream);
int asap_graph_end(void* stream, uint64_t* graph);
int asap_graph_launch(uint64_t graph, void* stream);
int asap_graph_release(uint64_t graph);

/* One job (replaces scheduler.py:387-436 run_job + FusedMoE + server.py:340-350 reply):
 * x/ids/w are the row's arena views (server.py:309-320 Row pointers); the token count comes from the
 * workspace's job descriptor. Routed experts [expert_base, expert_base+num_local) only, SwiGLU
 * h = silu(x W1^T) * (x W3^T) (clamped to +-swiglu_limit when swiglu_limit > 0), MXFP8 activations for MXFP4
 * experts and E4M3 activations with fp32 scales per 1 x 128 for FP8 experts (asap_experts_register_fp8),
 * out[t] = sum_j w[t,j] * (h W2^T), bf16, written to reply_seg row t; then done flag = seq (release, system
 * scope) at reply_done. reply_done == 0 skips the flag. */
int asap_ffn_job(uint64_t experts_handle, uint64_t ws_handle, uint64_t x, uint64_t ids, uint64_t w,
                 uint64_t reply_seg, uint64_t reply_done, float swiglu_limit, uint64_t status,
                 uint64_t timeout_ns, void* stream);

/* One message's arena views and reply target (asap_ffn_job's x/ids/w/reply_seg/reply_done). */
typedef struct {
  uint64_t x, ids, w, reply_seg, reply_done;
} asap_ffn_row_t;

/* asap_ffn_job over the `rows` messages of a joined job (their tokens numbered in row order); each row's reply goes
 * to its own segment and done flag (= that row's seq). */
int asap_ffn_job_rows(uint64_t experts_handle, uint64_t ws_handle, int32_t rows, const asap_ffn_row_t* row_views,
                      float swiglu_limit, uint64_t status, uint64_t timeout_ns, void* stream);

/* asap_ffn_job_rows whose reduce + reply (the reference's FfnServer.reply, server.py:340-350) runs on
 * `reply_stream` with `reply_ctas` CTAs, after an event behind GEMM2, while `stream` goes on to the next job with
 * persistent GEMM grids of `gemm_ctas` CTAs (fewer than the SMs leaves SMs free for the reply).  Across GPUs the
 * reply's stores cross NVLink, and this lets them overlap the next message's GEMMs.  The reply still reads this
 * workspace: a caller must not start another job on it before the reply is done (an event recorded on
 * `reply_stream` after this call), so consecutive jobs alternate between two workspaces. */
int asap_ffn_job_rows_overlap(uint64_t experts_handle, uint64_t ws_handle, int32_t rows,
                              const asap_ffn_row_t* row_views, float swiglu_limit, uint64_t status,
                              uint64_t timeout_ns, void* stream, void* reply_stream, int32_t gemm_ctas,
                              int32_t reply_ctas);

/* Per-kernel timing of asap_ffn_job on this workspace: when enabled, CUDA events are recorded on the job's
 * stream around its 5 stages (routing, quantise+permute, gemm1, gemm2, reduce+reply); last_timing waits
 * for the recorded jobs (the last 64 since enable) and returns each kernel's mean duration in ms (n >= 5). */
int asap_ffn_enable_timing(uint64_t ws_handle, int32_t enable);
int asap_ffn_last_timing(uint64_t ws_handle, float* ms, int32_t n);

/* Read back the job descriptor (debug/measurement): n, layer, seq, epoch, valid, the globaltimer (ns) at which
 * asap_ffn_wait saw the doorbell (0 when the job was posted by the host) and the one at which the reply's done
 * flag was released. Synchronizes `stream`. */
int asap_ffn_job_info(uint64_t ws_handle, int32_t* n, int32_t* layer_id, uint32_t* seq, int32_t* epoch,
                      int32_t* valid, uint64_t* t_seen_ns, uint64_t* t_reply_ns, void* stream);

/* Per-local-expert token-pair counts of the last job (int32 [num_local]) and the expert-major
 * permutation (int32 [n, topk] permuted row of pair (t, j), -1 when not local). Debug/tests; these are
 * device addresses inside the workspace, valid until the next job. */
int asap_ffn_debug_ptrs(uint64_t ws_handle, uint64_t* expert_counts, uint64_t* pair_pos, uint64_t* xq,
                        uint64_t* xq_sf, uint64_t* hq, uint64_t* hq_sf, uint64_t* y2);

#ifdef __cplusplus
}
#endif
#endif /* ASAP_H_ */
