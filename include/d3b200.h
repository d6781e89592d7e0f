/*
 * d3b200 -- B200 (sm_100a) routed-MoE expert offload hot path, C ABI.
 *
 * One shared library (libd3b200.so) with plain C entry points: raw pointers,
 * sizes and a CUDA stream, an int status return (D3_OK == 0, negative on
 * error), no exceptions across the ABI and no device or host allocation inside
 * any call.  Every launch goes on the caller's stream, issues no host sync and
 * keeps a static launch shape, so every call below (except d3_device_ptr_of,
 * which queries the driver) can be recorded into a CUDA graph and replayed;
 * device-side tables are read at replay time, never baked at capture.
 *
 * Device pointers: int32/int64 tables and byte buffers allocated by the caller
 * (e.g. torch tensors).  Host expert storage must be page-locked and mapped
 * (cudaHostAlloc / torch pin_memory); pass the pointer d3_device_ptr_of gives.
 *
 * Each entry point names the reference interface it replaces
 * (darth-feir/drama3-offloading, path:line).
 */
#ifndef D3B200_H
#define D3B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define D3_API __attribute__((visibility("default")))
#else
#define D3_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t, passed as an opaque pointer (0 = legacy default stream). */
typedef void* d3_stream_t;

enum {
  D3_OK = 0,
  D3_ERR_INVALID_ARG = -1,   /* bad size, null pointer, out-of-range parameter */
  D3_ERR_NOT_PINNED = -2,    /* host pointer is not page-locked / not mapped */
  D3_ERR_MISALIGNED = -3,    /* pointer or byte count not 16-byte aligned */
  D3_ERR_CUDA = -4,          /* a CUDA runtime/driver call failed (see d3_last_error) */
  D3_ERR_UNSUPPORTED = -5,   /* shape or device not supported by this build */
  D3_ERR_TOO_LARGE = -6,     /* exceeds a documented maximum */
  D3_ERR_WORKSPACE = -7      /* workspace pointer null or smaller than required */
};

/* Human-readable name of a status code (static string). */
D3_API const char* d3_status_string(int status);
/* Message of the last failing call on this host thread ("" if none). */
D3_API const char* d3_last_error(void);
/* ABI version: bumped on any incompatible change of these declarations. */
D3_API int d3_abi_version(void);

/* ------------------------------------------------------------------ fetch */

/* Device-visible address of page-locked host memory [host, host+bytes).
 * Fails with D3_ERR_NOT_PINNED for pageable memory.
 * Replaces device_ptr_of(at::Tensor) -- csrc/fetch_experts.cu:40-47. */
D3_API int d3_device_ptr_of(const void* host, size_t bytes, void** dev_out);

/* Copy expert idx[j] (expert_bytes each, from src_dev_base) into cache slot
 * slot[j] of dst for every j < *njobs (njobs is read on the device at run
 * time; launched as max_jobs x blocks_per_job CTAs of `threads` threads, the
 * surplus retiring without writing).  Requires 16-byte aligned src, dst and
 * expert_bytes, threads == 256.
 * Replaces fetch_experts(...) -- csrc/fetch_experts.cu:76-94; the semantics
 * of _fetch_experts -- bin/devcache.py:101-130. */
D3_API int d3_fetch_experts(const void* src_dev_base, void* dst, const int32_t* idx,
                     const int32_t* slot, const int32_t* njobs, int64_t expert_bytes,
                     int32_t max_jobs, int32_t blocks_per_job, int32_t threads,
                     d3_stream_t stream);

/* --------------------------------------------------------------- allocator */

/* One LRU resolve of k expert ids into cache slots, exactly the semantics of
 * _resolve_slots -- bin/devcache.py:45-98: step is bumped on the device; for
 * each id in order a hit keeps its slot, a miss takes the slot with the
 * smallest stamp (lowest index on ties), clears the victim's slot_of entry and
 * queues (fetch_slot, fetch_expert); every used slot is stamped with the new
 * step; *nmiss receives the number of queued fetches.  ids are int32
 * (ids_bytes == 4) or int64 (ids_bytes == 8, e.g. torch.topk output).
 * Ids outside [0, num_experts) get out_slot = -1 and are not fetched.
 * Limits: 1 <= k <= 64, 1 <= capacity <= 8192. */
D3_API int d3_resolve_slots(const void* ids, int32_t ids_bytes, int32_t k, int32_t* slot_of,
                     int32_t num_experts, int32_t* slot_expert, int64_t* stamp,
                     int32_t capacity, int32_t* out_slot, int32_t* fetch_slot,
                     int32_t* fetch_expert, int32_t* nmiss, int64_t* step,
                     d3_stream_t stream);

enum { D3_POLICY_LRU = 0, D3_POLICY_LFU = 1 };
enum { D3_MAX_BUFFERS = 4 };

/* One layer's device expert cache: the tables init_dev_cache allocates
 * (bin/devcache.py:146-167) plus the per-buffer host/cache byte layout
 * _copy_pairs describes (bin/devcache.py:170-181).  Plain data, filled by the
 * caller; the library never stores it. */
typedef struct d3_layer_cache {
  int32_t num_experts;      /* E */
  int32_t capacity;         /* C slots */
  int32_t policy;           /* D3_POLICY_LRU or D3_POLICY_LFU */
  int32_t nbuf;             /* buffers per expert, 1..D3_MAX_BUFFERS */
  int32_t* slot_of;         /* [E]  expert -> slot or -1 */
  int32_t* slot_expert;     /* [C]  slot -> expert or -1 */
  int64_t* stamp;           /* [C]  step of last use */
  int64_t* step;            /* [1]  call counter, bumped on device */
  int64_t* freq;            /* [C]  LFU: uses since insertion (NULL for LRU) */
  int64_t* ins;             /* [C]  LFU: insertion sequence (NULL for LRU) */
  int32_t* out_slot;        /* [k]  resolved slot per id */
  int32_t* fetch_slot;      /* [k]  queued fetch: destination slot */
  int32_t* fetch_expert;    /* [k]  queued fetch: expert id */
  int32_t* nmiss;           /* [1]  queued fetch count */
  int64_t* counters;        /* [4]  cumulative {calls, hits, misses, bytes fetched}, or NULL */
  const void* host[D3_MAX_BUFFERS];  /* device-visible pinned host base, [E][bytes[b]] */
  void* cache[D3_MAX_BUFFERS];       /* device cache buffer, [C][bytes[b]] */
  int64_t bytes[D3_MAX_BUFFERS];     /* bytes per expert of buffer b (multiple of 16) */
} d3_layer_cache;

/* Resolve k ids through layer->policy and fetch every miss's nbuf buffers from
 * pinned host memory into its slot: one allocator launch and one fetch launch
 * (a fixed grid of fetch_ctas CTAs; 0 = one per SM), dependent via
 * programmatic launch.  Results: layer->out_slot[0..k).
 * Replaces dev_resolve_and_fetch -- bin/devcache.py:230-255 (which issues
 * _resolve_slots plus four fetch launches). */
D3_API int d3_resolve_fetch(const d3_layer_cache* layer, const void* ids, int32_t ids_bytes,
                     int32_t k, int32_t fetch_ctas, d3_stream_t stream);

/* One decode row (T = 1, k ids) through the layer's cache with the fetch and
 * the expert compute overlapped: the allocator launch (as d3_resolve_fetch),
 * then ONE launch in which fetch_ctas CTAs (0 = 64) move the misses -- the
 * W13/S13 bytes of every job first -- while the other CTAs run the gate/up
 * products of the resident experts and of the optional shared expert, then
 * those of each fetched expert after a bounded wait (2 s; *err_word = 41 on
 * expiry) until its job's W13/S13 bytes have landed; then the down projection
 * into out (bf16 [1, H], added when accumulate).  layer: the 4 buffers w13
 * [C][2I][H] e4m3, w2 [C][H][I], s13 [C][2I/128][H/128] f32, s2
 * [C][H/128][I/128] f32, capacity >= k; H, I as for the decode path of
 * d3_moe_fp8_forward_shared (multiples of 512).  workspace: at least
 * d3_resolve_fetch_moe_workspace_size(k, H, I) bytes, 16-byte aligned.  Same
 * slot tables and the same output bits as d3_resolve_fetch followed by
 * d3_moe_fp8_forward(_shared) over the cache.  Replaces the reference's decode
 * step of dev_cached_forward (bin/devcache.py:258-277: dev_resolve_and_fetch,
 * then fp8_moe_forward over the cache).  stages: a mask of the launches to
 * issue -- 1 allocator, 2 fetch + gate/up, 4 down projection; 7 = all of it
 * (same arguments and workspace for the split calls, in that order; for
 * timing the launches apart). */
D3_API size_t d3_resolve_fetch_moe_workspace_size(int32_t k, int32_t H, int32_t I);
D3_API int d3_resolve_fetch_moe(const d3_layer_cache* layer, const void* ids, int32_t ids_bytes,
                                int32_t k, const void* x, const void* weights,
                                int32_t weights_f32, int32_t H, int32_t I,
                                const void* shared_w13, const void* shared_w2,
                                const void* shared_gate, void* out, int32_t accumulate,
                                int32_t* err_word, void* workspace, size_t workspace_bytes,
                                int32_t fetch_ctas, int32_t stages, d3_stream_t stream);

/* d3_resolve_fetch_moe plus L2 warm windows: while the fetch holds the host
 * link, the gate/up CTAs that have finished hint the n_windows (<= 4) ranges
 * [l2_warm[w], l2_warm[w] + l2_warm_bytes[w]) into L2 (whole 128-byte lines;
 * a hint, never waited on).  Meant for static weights the next launches read
 * (the next layer's router gate and first dense weight), which HBM, idle
 * during the host-bound fetch, then serves from L2.  The two arrays are host
 * memory, read during the call.  No counterpart in the reference. */
D3_API int d3_resolve_fetch_moe_l2warm(const d3_layer_cache* layer, const void* ids,
                                       int32_t ids_bytes, int32_t k, const void* x,
                                       const void* weights, int32_t weights_f32, int32_t H,
                                       int32_t I, const void* shared_w13, const void* shared_w2,
                                       const void* shared_gate, void* out, int32_t accumulate,
                                       int32_t* err_word, void* workspace, size_t workspace_bytes,
                                       int32_t fetch_ctas, int32_t stages,
                                       const void* const* l2_warm, const size_t* l2_warm_bytes,
                                       int32_t n_windows, d3_stream_t stream);

/* Only the fetch half of d3_resolve_fetch: copy the jobs already queued in
 * layer->fetch_slot / fetch_expert / *nmiss (e.g. by d3_resolve_slots or a
 * host-written job list) for all nbuf buffers, one launch of fetch_ctas CTAs
 * (0 = one per SM).  The device job count may be 0..C; no allocator runs.
 * Replaces the four per-buffer fetch launches of dev_resolve_and_fetch --
 * bin/devcache.py:240-254. */
D3_API int d3_fetch_jobs(const d3_layer_cache* layer, int32_t fetch_ctas, d3_stream_t stream);

/* Read-only lookup (no stamp, no insert): slot_out[i] = slot_of[ids[i]] or -1.
 * The prefill path's borrow from the device cache -- bin/offload.py:195-214. */
D3_API int d3_lookup_slots(const int32_t* slot_of, int32_t num_experts, const void* ids,
                    int32_t ids_bytes, int32_t n, int32_t* slot_out, d3_stream_t stream);

/* Prefill plan, without a host sync: the distinct experts a batch routes to.
 * expert_list[0..*n_distinct) = those experts ascending, remap[e] = their
 * compact index (-1 if unused), local_ids[i] = remap[ids[i]] (-1 for
 * out-of-range ids).  One launch.
 * Replaces torch.unique(topk_ids.cpu(), return_inverse=True) of the gather
 * path -- bin/offload.py:157-158 (a host sync per layer). */
D3_API int d3_prefill_plan(const void* ids, int32_t ids_bytes, int32_t n_pairs,
                           int32_t num_experts, int32_t* expert_list, int32_t* n_distinct,
                           int32_t* remap, int32_t* local_ids, d3_stream_t stream);

/* Gather the experts of expert_list[0..*n_distinct) into compact buffers
 * dst[b] ([n_max][layer->bytes[b]]) in one launch: an expert resident in the
 * layer's device cache (layer->slot_of[e] >= 0) is copied from its slot --
 * read-only, no stamp or insert -- any other is read from the pinned host
 * store.  counters (optional, int64[2]) accumulate {borrowed, fetched}.
 * layer->slot_of may be NULL (no cache: everything from host).
 * Replaces the hybrid gather of offloaded_forward -- bin/offload.py:186-226
 * (per-expert copy_ calls plus index copies of the scales). */
D3_API int d3_gather_experts(const d3_layer_cache* layer, const int32_t* expert_list,
                             const int32_t* n_distinct, void* const* dst, int64_t* counters,
                             int32_t fetch_ctas, d3_stream_t stream);

/* ------------------------------------------------------------------ router */

/* Workspace bytes d3_router_topk needs for T tokens and E experts. */
D3_API size_t d3_router_workspace_size(int32_t T, int32_t E);

/* MoE router: logits = x @ gate_w^T (bf16 [T,H] x bf16 [E,H]), softmax over E,
 * top-k (ties -> lower expert index), weights renormalised over the k when
 * renorm != 0.  Logits are the exactly rounded bf16 of each dot product.
 * Outputs: ids_out int32 [T,k]; weights_out f32 [T,k] and/or
 * weights_bf16_out bf16 [T,k] (either may be NULL).  The workspace must be
 * zero-filled once before its first use (every call leaves it reusable, for
 * any T).  Limits: T <= 65536, H % 8 == 0, H <= 8192, E <= 1024, k <= 32.
 * Replaces the upstream MoE block's gate -> softmax -> topk -> renorm
 * (fish-speech moe.py:217-220, quoted at notes/01-static-findings.md:133-138),
 * whose topk_ids feed dev_cached_forward -- bin/devcache.py:258-277. */
D3_API int d3_router_topk(const void* x, const void* gate_w, int32_t T, int32_t H, int32_t E,
                          int32_t topk, int32_t renorm, int32_t* ids_out, float* weights_out,
                          void* weights_bf16_out, void* workspace, size_t workspace_bytes,
                          d3_stream_t stream);

/* d3_router_topk without a workspace argument, for callers that cannot
 * allocate device memory (a runtime that binds only this C ABI and has no
 * device allocator, a serving loop that must never allocate or risk an
 * out-of-memory error mid-decode, a process whose free device memory all went
 * to the expert cache).  No counterpart in the reference; it allocates
 * nothing.  Same inputs, outputs and results as d3_router_topk.
 * Scratch: a fixed array of 1 KiB + 256 KiB inside the library, reserved on
 * every GPU that loads it until the process exits.  Limits: T <= 2048 and
 * T * E <= 65536 (e.g. T = 256 at E = 256); larger calls return
 * D3_ERR_TOO_LARGE.  The first call on each device looks the array's device
 * address up and zeroes its counters (a synchronous memset), so make it
 * before any stream capture on that device.  All
 * calls share the one array, so calls that overlap on the GPU (different
 * streams, or concurrent graphs) race: serialise them. */
D3_API int d3_router_topk_noalloc(const void* x, const void* gate_w, int32_t T, int32_t H,
                                  int32_t E, int32_t topk, int32_t renorm, int32_t* ids_out,
                                  float* weights_out, void* weights_bf16_out, d3_stream_t stream);

/* ------------------------------------------------------------- expert GEMM */

/* Workspace bytes d3_moe_fp8_forward needs (0 = unsupported shape). */
D3_API size_t d3_moe_workspace_size(int32_t T, int32_t topk, int32_t n_experts, int32_t H,
                                    int32_t I);

/* Routed MoE over block-scaled FP8 experts.  For every pair (t, j) with
 * e = ids[t,j] in [0, n_experts):
 *   h = silu(x_t Wg[e]^T) * (x_t Wu[e]^T),   out_t += weights[t,j] * h Wd[e]^T
 * x bf16 [T,H]; ids int32/int64 [T,topk] (ids_bytes 4/8; out-of-range ids are
 * skipped); weights f32 (weights_f32 = 1) or bf16 [T,topk]; w13 e4m3 [n,2I,H]
 * (gate rows [0,I), up rows [I,2I)), s13 f32 [n,2I/128,H/128]; w2 e4m3 [n,H,I],
 * s2 f32 [n,H/128,I/128] (weight = byte x scale of its 128x128 block);
 * out bf16 [T,H], overwritten, or with accumulate != 0 added to (out may then
 * alias x: the residual add of the MoE block).  err_word: device int32, set
 * non-zero (never cleared) if a kernel gave up on a bounded wait.
 * Limits: H, I multiples of 128 in
 * [128, 16384]; T*topk <= 65536; n_experts <= 8192.
 * Replaces upstream fp8_moe_forward(x, ids, w, w13, s13, w2, s2) as called by
 * dev_cached_forward -- bin/devcache.py:275-277 -- and the gather paths --
 * bin/offload.py:177, :239, :340, :388, :449. */
D3_API int d3_moe_fp8_forward(const void* x, const void* ids, int32_t ids_bytes,
                              const void* weights, int32_t weights_f32, int32_t T, int32_t topk,
                              const void* w13, const float* s13, const void* w2, const float* s2,
                              int32_t n_experts, int32_t H, int32_t I, void* out,
                              int32_t accumulate, int32_t* err_word, void* workspace,
                              size_t workspace_bytes, d3_stream_t stream);

/* d3_moe_fp8_forward plus Drama-3's shared expert in the same two launches:
 * every token also runs the bf16 SwiGLU expert shared_w13 [2I, H] (gate rows
 * [0, I), up rows [I, 2I)), shared_w2 [H, I], scaled by
 * sigmoid(x . shared_gate) (shared_gate [H] bf16; null = ungated), all added
 * into out.  Decode batches only (T * topk <= 32, H and I multiples of 512);
 * larger batches -> D3_ERR_UNSUPPORTED (run the shared expert as a plain
 * dense GEMM).  The upstream MoE block computes the shared expert with its
 * own bf16 Linear layers outside the offloaded path (notes/01-static-
 * findings.md:80-82; shared_expert_gate: notes/drama3-config.json:215). */
D3_API int d3_moe_fp8_forward_shared(const void* x, const void* ids, int32_t ids_bytes,
                                     const void* weights, int32_t weights_f32, int32_t T,
                                     int32_t topk, const void* w13, const float* s13,
                                     const void* w2, const float* s2, int32_t n_experts,
                                     int32_t H, int32_t I, const void* shared_w13,
                                     const void* shared_w2, const void* shared_gate, void* out,
                                     int32_t accumulate, int32_t* err_word, void* workspace,
                                     size_t workspace_bytes, d3_stream_t stream);

/* ---------------------------------------------------- expert parallelism */

/* Build the static-capacity all-to-all send buffer for expert parallelism
 * (experts e in [d*experts_per_rank, (d+1)*experts_per_rank) live on rank d).
 * Pair (t, j) with expert e = ids[t,j] goes to row d*cap + r of send_x
 * [n_ranks*cap, H] bf16 (r = its rank among the pairs bound for d, in pair
 * order) with send_eid[row] = e - d*experts_per_rank; unused rows get -1;
 * src_slot[t,j] = row (-1 if e is out of range or d's block is full, counted
 * in *overflow).  cap = T*topk never overflows.  No counterpart in the
 * reference (it has no multi-GPU path); the resident expert-parallel
 * configuration of the B200 build. */
D3_API int d3_ep_dispatch_pack(const void* x, const int32_t* ids, int32_t T, int32_t topk,
                               int32_t H, int32_t n_ranks, int32_t experts_per_rank, int32_t cap,
                               void* send_x, int32_t* send_eid, int32_t* src_slot,
                               int32_t* overflow, d3_stream_t stream);

/* out[t] (+)= sum_j weights[t,j] * ret[src_slot[t,j]] (bf16 rows of H, fixed
 * j order, skipped where src_slot < 0): the combine after the return
 * all-to-all.  weights f32 (weights_f32 = 1) or bf16.  No counterpart in the
 * reference. */
D3_API int d3_ep_combine(const void* ret, const int32_t* src_slot, const void* weights,
                         int32_t weights_f32, int32_t T, int32_t topk, int32_t H, void* out,
                         int32_t accumulate, d3_stream_t stream);

/* ---------------------------------------------------------------- NVLink exchange (EP) */

/* CUDA IPC of the allocation that holds `ptr`: a 64-byte handle plus ptr's
 * offset inside it (d3_ipc_open in another process maps the allocation; add
 * the offset).  For the expert-parallel exchange buffers. */
D3_API int d3_ipc_get(const void* ptr, void* handle, uint64_t* offset);
D3_API int d3_ipc_open(const void* handle, void** base);
D3_API int d3_ipc_close(void* base);

/* The expert-parallel dispatch over peer memory: the same packing as
 * d3_ep_dispatch_pack, but each token row and local expert id is stored
 * straight into its destination rank's exchange buffer (peer_recv_x[d],
 * peer_recv_eid[d]: rows [rank*cap, (rank+1)*cap) belong to this source),
 * then flag_d[rank] = epoch is released on every destination (*epoch is a
 * device counter this call increments once).  counter: a device uint32 that
 * is zero between calls.  n_ranks <= 16; T * topk <= 4096 (D3_ERR_TOO_LARGE
 * beyond: larger batches take d3_ep_dispatch_pack and an all-to-all).  No
 * counterpart in the reference. */
D3_API int d3_ep_dispatch_p2p(const void* x, const int32_t* ids, int32_t T, int32_t topk,
                              int32_t H, int32_t n_ranks, int32_t rank,
                              int32_t experts_per_rank, int32_t cap, void* const* peer_recv_x,
                              int32_t* const* peer_recv_eid, int64_t* const* peer_flag_d,
                              int32_t* src_slot, int32_t* overflow, int64_t* epoch,
                              uint32_t* counter, d3_stream_t stream);

/* The return path: every received row with a valid expert id (recv_eid, local)
 * goes from y (local expert outputs, [n_ranks*cap, H]) into its source rank's
 * ret rows [rank*cap, ...), then flag_r[rank] = *epoch on every source. */
D3_API int d3_ep_return_p2p(const void* y, const int32_t* recv_eid, int32_t n_ranks,
                            int32_t rank, int32_t cap, int32_t H, void* const* peer_ret,
                            int64_t* const* peer_flag_r, const int64_t* epoch, uint32_t* counter,
                            d3_stream_t stream);

/* One warp waits until flags[r] >= *epoch for every r < n_ranks (system-scope
 * acquire loads), at most budget_ns of GPU time; on expiry *err_word = code
 * (if it was 0) and the kernel returns. */
D3_API int d3_ep_wait(const int64_t* flags, int32_t n_ranks, const int64_t* epoch,
                      int32_t* err_word, int32_t code, int64_t budget_ns, d3_stream_t stream);

/* The expert call of one expert-parallel layer with the NVLink exchange folded
 * into its first and last launches: d3_moe_fp8_forward over the received rows
 * (x = recv_x [T = n_ranks*cap, H], ids = recv_eid, topk normally 1), whose
 * route launch first waits (bounded, budget_ns; on expiry *err_word =
 * wait_code) until wait_flags[r] >= *epoch for every rank r, and whose combine
 * launch stores each served row t = s*cap + j straight into row rank*cap + j
 * of source s's return buffer (peer_ret[s]), then publishes
 * peer_flag_r[s][rank] = *epoch on every source.  counter: a device uint32,
 * zero between calls.  Always the tensor-core path; no accumulate.  Replaces
 * d3_ep_wait + d3_moe_fp8_forward + d3_ep_return_p2p.  No counterpart in the
 * reference. */
D3_API int d3_moe_fp8_forward_p2p(const void* x, const void* ids, int32_t ids_bytes,
                                  const void* weights, int32_t weights_f32, int32_t T,
                                  int32_t topk, const void* w13, const float* s13, const void* w2,
                                  const float* s2, int32_t n_experts, int32_t H, int32_t I,
                                  int32_t* err_word, void* workspace, size_t workspace_bytes,
                                  const int64_t* wait_flags, const int64_t* epoch,
                                  int32_t n_ranks, int32_t rank, int32_t cap,
                                  void* const* peer_ret, int64_t* const* peer_flag_r,
                                  uint32_t* counter, int32_t wait_code, int64_t budget_ns,
                                  d3_stream_t stream);

/* d3_ep_combine after a bounded wait (as d3_ep_wait) until flag_r[r] >= *epoch
 * for every serving rank r: replaces d3_ep_wait + d3_ep_combine. */
D3_API int d3_ep_combine_p2p(const void* ret, const int32_t* src_slot, const void* weights,
                             int32_t weights_f32, int32_t T, int32_t topk, int32_t H, void* out,
                             int32_t accumulate, const int64_t* flag_r, int32_t n_ranks,
                             const int64_t* epoch, int32_t* err_word, int32_t code,
                             int64_t budget_ns, d3_stream_t stream);

/* ---------------------------------------------------------------- routing census / trace */

/* counts[e] += occurrences of expert e among the rows*k ids (int32 or int64,
 * ids_bytes 4 or 8; ids outside [0, num_experts) are not counted); a call of
 * exactly one row (a decode step) also adds to counts_decode when that is
 * non-null.  counts / counts_decode: this layer's int64 [num_experts] rows of
 * the census.  Device-side, sync-free and graph-capturable.  Replaces the
 * reference's host-side census (bin/offload.py:257-287 enable_census / _count,
 * which copies the ids to the CPU on every call). */
D3_API int d3_census_add(const void* ids, int32_t ids_bytes, int32_t rows, int32_t k,
                         int32_t num_experts, int64_t* counts, int64_t* counts_decode,
                         d3_stream_t stream);

/* Router trace: appends one record per row to a device ring of `capacity`
 * records of 3 + k int32 each: {first row index of this call (low 31 bits of
 * the cursor), layer, phase (1 if the call has exactly one row -- decode --
 * else 0), ids[k]}.  *cursor (int64, device) counts every row ever appended;
 * record r lives at ring[(r % capacity) * (3 + k)].  rows > capacity ->
 * D3_ERR_TOO_LARGE.  Replaces bin/offload.py:40-79 RouterTrace.add (host
 * lists, a device sync per call). */
D3_API int d3_trace_append(const void* ids, int32_t ids_bytes, int32_t rows, int32_t k,
                           int32_t layer, int32_t* ring, int64_t* cursor, int64_t capacity,
                           d3_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* D3B200_H */
