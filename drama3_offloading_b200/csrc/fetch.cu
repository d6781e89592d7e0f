// Expert fetch (pinned host -> device cache slots) and the device slot allocator.
//
// Replaces the reference's csrc/fetch_experts.cu (fetch_kernel :49-69, host
// wrapper :76-94, device_ptr_of :40-47) and bin/devcache.py's Triton
// _resolve_slots (:45-98) / _fetch_experts (:101-130) / dev_resolve_and_fetch
// (:230-255).
//
// Why a kernel and not a memcpy: a captured cudaMemcpyAsync bakes its source
// address, so a replayed graph would keep copying the capture-time expert.
// These kernels read the job table (which expert, which slot, how many) from
// device memory when they run, so one captured graph serves whatever the
// router picks on each replay.
//
// B200 design:
//  * The allocator is one warp: the victim search (argmin of C stamps, lowest
//    index on ties) is a warp-parallel scan over a shared-memory copy of the
//    stamps plus a shuffle reduction, instead of the reference's serial O(k*C)
//    single-thread loop.  Decisions stay sequential over the k ids, exactly as
//    the reference orders them.
//  * The fetch moves all buffers of all missed experts in ONE launch with a
//    fixed grid (one CTA per SM by default): the jobs' bytes form one flat
//    range that every CTA strides over, so even a single miss is spread over
//    the whole grid and keeps enough 512-byte warp requests in flight to fill
//    the host link.  Loads are 16-byte vector loads of mapped host memory that
//    bypass L1; stores are plain (the GEMM reads the slot from L2 next).
//  * The fetch launch depends on the allocator launch programmatically
//    (griddepcontrol), so its CTAs are resident before the allocator ends.

#include "d3_common.cuh"
#include "fetch_flat.cuh"

#include <stdlib.h>
#include <string.h>

namespace d3 {

// ---------------------------------------------------------------- status

static thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(D3_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) v = getenv("D3_NO_PDL") ? 0 : 1;
  return v == 1;
}

// ---------------------------------------------------------------- kernels

// Reference-compatible per-buffer fetch: grid (blocks_per_job, max_jobs).
// Job j copies expert idx[j] into slot[j]; CTAs of jobs >= *njobs retire.
__global__ void __launch_bounds__(256) fetch_jobs_kernel(const uint4* __restrict__ src,
                                                         uint4* __restrict__ dst,
                                                         const int32_t* __restrict__ idx,
                                                         const int32_t* __restrict__ slot,
                                                         const int32_t* __restrict__ njobs,
                                                         int64_t vec_per_expert) {
  const int j = blockIdx.y;
  if (j >= *njobs) return;
  const uint4* s = src + (int64_t)idx[j] * vec_per_expert;
  uint4* d = dst + (int64_t)slot[j] * vec_per_expert;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // four independent 16-byte loads in flight per thread before any store
  for (; i + 3 * stride < vec_per_expert; i += 4 * stride) {
    uint4 a = ld_stream_u4(s + i), b = ld_stream_u4(s + i + stride);
    uint4 c = ld_stream_u4(s + i + 2 * stride), e = ld_stream_u4(s + i + 3 * stride);
    d[i] = a;
    d[i + stride] = b;
    d[i + 2 * stride] = c;
    d[i + 3 * stride] = e;
  }
  for (; i < vec_per_expert; i += stride) d[i] = ld_stream_u4(s + i);
}

// Flat multi-buffer fetch: the byte range of job j / buffer b / vector v is
// linearised as j*vec_total + (prefix_b + v); CTAs stride over chunks of
// kFetchThreads*kFetchUnroll vectors (16 KiB).
__global__ void __launch_bounds__(kFetchThreads) fetch_layer_kernel(FetchParams p) {
  pdl_wait();  // the allocator's job table must be complete
  const int nm = *p.nmiss;
  if (nm <= 0) return;
  const int64_t total = (int64_t)nm * p.vec_total;
  constexpr int64_t kChunk = (int64_t)kFetchThreads * kFetchUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kChunk; base < total;
       base += (int64_t)gridDim.x * kChunk) {
    uint4 v[kFetchUnroll];
    uint4* dptr[kFetchUnroll];
#pragma unroll
    for (int u = 0; u < kFetchUnroll; ++u) {
      const int64_t g = base + (int64_t)u * kFetchThreads + threadIdx.x;
      dptr[u] = nullptr;
      if (g < total) {
        const int64_t j = g / p.vec_total;
        int64_t r = g - j * p.vec_total;
        int b = 0;
        while (b < p.nbuf - 1 && r >= p.vecs[b]) { r -= p.vecs[b]; ++b; }
        const int64_t e = p.fetch_expert[j], s = p.fetch_slot[j];
        v[u] = ld_stream_u4(p.host[b] + e * p.vecs[b] + r);
        dptr[u] = p.cache[b] + s * p.vecs[b] + r;
      }
    }
#pragma unroll
    for (int u = 0; u < kFetchUnroll; ++u)
      if (dptr[u]) *dptr[u] = v[u];
  }
}

struct ResolveParams {
  const void* ids;
  int32_t ids_bytes;
  int32_t k;
  int32_t num_experts;
  int32_t capacity;
  int32_t policy;
  int32_t* slot_of;
  int32_t* slot_expert;
  int64_t* stamp;
  int64_t* step;
  int64_t* freq;
  int64_t* ins;
  int32_t* out_slot;
  int32_t* fetch_slot;
  int32_t* fetch_expert;
  int32_t* nmiss;
  int64_t* counters;
  int64_t expert_bytes;
  int64_t* zero;       // [nzero] cleared by this launch (the overlap launch's counters)
  int32_t nzero;
  int32_t slot_of_smem;  // stage the whole slot_of table in shared memory (1) or look it up (0)
};

__device__ __forceinline__ int32_t load_id(const void* ids, int bytes, int i) {
  if (bytes == 8) {
    const int64_t v = static_cast<const int64_t*>(ids)[i];
    return (v < INT32_MIN || v > INT32_MAX) ? -1 : (int32_t)v;
  }
  return static_cast<const int32_t*>(ids)[i];
}

// Lexicographic (key, index) minimum across the warp.
__device__ __forceinline__ void warp_argmin(int64_t& key, int& idx) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const int64_t ok = __shfl_xor_sync(0xffffffffu, key, off);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
    if (ok < key || (ok == key && oi < idx)) { key = ok; idx = oi; }
  }
}

// One warp.  LRU: the _resolve_slots decision sequence.  LFU: victim is the
// lexicographic min of (used this step, uses since insert, insertion seq).
// Every table read the decisions depend on is prefetched in parallel before
// the sequential loop (the k ids, their slot_of entries, the C stamps and
// slot owners into shared memory), so the loop itself touches only registers
// and shared memory; lane 0 streams the table updates out to global memory.
// A prefetched slot_of entry is still valid iff the slot's owner is still
// that expert; an id seen earlier in the same call resolves to the slot its
// latest occurrence got (again iff still owned) -- together exactly the
// reference's live slot_of lookup.
// Every prefetch load is issued before any is used (batched into registers),
// so the prefetch is one memory round trip: with slot_of_smem the whole
// slot_of table is staged alongside the ids instead of looked up by them.
// Dynamic shared memory: stamp[C] (+ freq[C], ins[C] for LFU) int64, then
// owner[C] int32, then (slot_of_smem) slot_of[num_experts] int32, then the
// fast path's marks[C] bytes.
__global__ void __launch_bounds__(32) resolve_kernel(ResolveParams p) {
  extern __shared__ int64_t sh[];
  const int C = p.capacity;
  const bool lfu = p.policy == D3_POLICY_LFU;
  int64_t* s_stamp = sh;
  int64_t* s_freq = sh + C;
  int64_t* s_ins = sh + 2 * C;
  int32_t* s_owner = reinterpret_cast<int32_t*>(sh + (lfu ? 3 : 1) * C);
  int32_t* s_slot_of = s_owner + C;
  const int lane = threadIdx.x;
  const unsigned full = 0xffffffffu;
  const int n = p.num_experts;
  pdl_trigger();  // the dependent fetch grid may start launching now
  // L2 prefetch hints for every line the prefetch below reads, issued while
  // the preceding launch (the router) still runs: a hint returns no data and
  // L2 is the point of coherence, so the loads after the wait still see that
  // launch's writes; what it saves is the DRAM and address-translation
  // latency of tables the layers in between have evicted.
  {
    auto hint = [&](const void* base, size_t bytes) {
      for (size_t o = (size_t)lane * 128; o < bytes; o += 32 * 128)
        prefetch_l2(static_cast<const char*>(base) + o);
    };
    hint(p.ids, (size_t)p.k * p.ids_bytes);
    hint(p.slot_of, (size_t)n * sizeof(int32_t));
    hint(p.stamp, (size_t)C * sizeof(int64_t));
    hint(p.slot_expert, (size_t)C * sizeof(int32_t));
    hint(p.step, sizeof(int64_t));
    if (lfu) { hint(p.freq, (size_t)C * sizeof(int64_t)); hint(p.ins, (size_t)C * sizeof(int64_t)); }
  }
  pdl_wait();     // ids may come from the launch just before this one
  // ---- parallel prefetch: the ids, the slot tables, the step
  int e_lo = -1, e_hi = -1, pre_lo = -1, pre_hi = -1;
  if (lane < p.k) e_lo = load_id(p.ids, p.ids_bytes, lane);
  if (lane + 32 < p.k) e_hi = load_id(p.ids, p.ids_bytes, lane + 32);
  const int64_t step = *p.step + 1;
  constexpr int kB = 8;  // loads per lane in flight per batch
  if (p.slot_of_smem) {
    for (int base = 0; base < n; base += 32 * kB) {
      int32_t v[kB];
#pragma unroll
      for (int u = 0; u < kB; ++u) {
        const int i = base + 32 * u + lane;
        v[u] = i < n ? p.slot_of[i] : -1;
      }
#pragma unroll
      for (int u = 0; u < kB; ++u) {
        const int i = base + 32 * u + lane;
        if (i < n) s_slot_of[i] = v[u];
      }
    }
  }
  for (int base = 0; base < C; base += 32 * kB) {
    int64_t st[kB];
    int32_t ow[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int c = base + 32 * u + lane;
      st[u] = c < C ? p.stamp[c] : 0;
      ow[u] = c < C ? p.slot_expert[c] : -1;
    }
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int c = base + 32 * u + lane;
      if (c < C) { s_stamp[c] = st[u]; s_owner[c] = ow[u]; }
    }
  }
  if (lfu)
    for (int c = lane; c < C; c += 32) { s_freq[c] = p.freq[c]; s_ins[c] = p.ins[c]; }
  if (e_lo >= n) e_lo = -1;
  if (e_hi >= n) e_hi = -1;
  if (!p.slot_of_smem) {
    if (e_lo >= 0) pre_lo = p.slot_of[e_lo];
    if (e_hi >= 0) pre_hi = p.slot_of[e_hi];
  }
  __syncwarp();  // the staged tables are visible to every lane
  if (p.slot_of_smem) {
    if (e_lo >= 0) pre_lo = s_slot_of[e_lo];
    if (e_hi >= 0) pre_hi = s_slot_of[e_hi];
  }
  for (int i = lane; i < p.nzero; i += 32) p.zero[i] = 0;
  // LRU victim search on 32-bit keys (two warp reductions) while every stamp
  // -- and the step the call writes -- fits in int32, which holds for the
  // first 2^31 calls of a layer; otherwise the 64-bit search
  bool fits = step <= (int64_t)INT32_MAX;
  for (int c = lane; c < C; c += 32)
    fits &= s_stamp[c] >= (int64_t)INT32_MIN && s_stamp[c] <= (int64_t)INT32_MAX;
  const bool key32 = __all_sync(full, fits);
  __syncwarp();
  int out_lo = -1, out_hi = -1;
  int nmiss = 0, hits = 0;
  // ---- LRU fast path (k <= 32 ids, one per lane; k < C; 32-bit keys): every
  // hit at once, then the misses' victims in id order by repeated warp
  // arg-min over the slots no hit of this call uses.  The sequential rule
  // gives a miss the oldest slot not touched BEFORE it; this gives it the
  // oldest slot not touched at all -- the same slot unless a slot hit later
  // in the call is older than a victim, which the check below detects (then
  // the sequential loop decides the call instead).  Duplicate ids take their
  // first occurrence's slot, as the sequential walk's later lookups do.
  bool fast_done = false;
  if (!lfu && key32 && p.k <= 32 && p.k < C) {
    uint8_t* s_mark = reinterpret_cast<uint8_t*>(s_slot_of + (p.slot_of_smem ? n : 0));  // [C]
    __shared__ int s_vict[32];
    const bool valid = lane < p.k && e_lo >= 0;
    const unsigned same = __match_any_sync(full, valid ? e_lo : -1 - lane);
    const int first = __ffs(same) - 1;
    const bool isfirst = valid && first == lane;
    const bool hit = isfirst && pre_lo >= 0 && s_owner[pre_lo] == e_lo;
    for (int c = lane; c < C; c += 32) s_mark[c] = 0;
    __syncwarp();
    if (hit) s_mark[pre_lo] = 1;
    __syncwarp();
    const unsigned missmask = __ballot_sync(full, isfirst && !hit);
    const int nm = __popc(missmask), nh = __popc(__ballot_sync(full, hit));
    bool ok = nm <= C - nh;
    int vkey = INT32_MIN, vidx = -1;   // the last (newest) victim's (stamp, slot)
    for (int r = 0; ok && r < nm; ++r) {
      int key = INT32_MAX, bi = INT32_MAX;
      for (int c = lane; c < C; c += 32) {
        const int v = (int)s_stamp[c];
        if (s_mark[c] == 0 && v < key) { key = v; bi = c; }
      }
      vkey = __reduce_min_sync(full, key);
      vidx = __reduce_min_sync(full, key == vkey ? bi : INT32_MAX);
      if (lane == 0) { s_vict[r] = vidx; s_mark[vidx] = 2; }
      __syncwarp();
    }
    if (ok && nm > 0) {
      bool conflict = false;
      if (hit) {
        const int hs = (int)s_stamp[pre_lo];
        conflict = hs < vkey || (hs == vkey && pre_lo < vidx);
      }
      ok = !__any_sync(full, conflict);
    }
    if (ok) {
      const int rank = __popc(missmask & ((1u << lane) - 1u));
      int s = hit ? pre_lo : (isfirst ? s_vict[rank] : -1);
      const int sf = __shfl_sync(full, s, first);
      if (valid && !isfirst) s = sf;
      if (lane < p.k) p.out_slot[lane] = s;
      if (isfirst) p.stamp[s] = step;
      if (isfirst && !hit) {
        const int32_t victim = s_owner[s];
        if (victim >= 0) p.slot_of[victim] = -1;
        p.slot_of[e_lo] = s;
        p.slot_expert[s] = e_lo;
        p.fetch_slot[rank] = s;
        p.fetch_expert[rank] = e_lo;
      }
      nmiss = nm;
      hits = __popc(__ballot_sync(full, valid)) - nm;
      fast_done = true;
    }
    __syncwarp();
  }
  for (int i = 0; i < p.k && !fast_done; ++i) {
    const int src = i & 31;
    const int32_t e = __shfl_sync(full, i < 32 ? e_lo : e_hi, src);
    int32_t s = __shfl_sync(full, i < 32 ? pre_lo : pre_hi, src);
    if (e < 0) {
      if (lane == 0) p.out_slot[i] = -1;
      continue;  // out_lo/out_hi stay -1 for this i
    }
    if (s >= 0 && s_owner[s] != e) s = -1;  // evicted earlier in this call
    if (s < 0) {
      // latest earlier occurrence of e in this call
      const unsigned m_lo = __ballot_sync(full, lane < i && e_lo == e);
      const unsigned m_hi = __ballot_sync(full, lane + 32 < i && e_hi == e);
      const int j = m_hi ? 32 + (31 - __clz(m_hi)) : (m_lo ? 31 - __clz(m_lo) : -1);
      const int sj = __shfl_sync(full, j >= 32 ? out_hi : out_lo, j >= 0 ? (j & 31) : 0);
      if (j >= 0 && sj >= 0 && s_owner[sj] == e) s = sj;
    }
    if (s < 0) {
      int best = 0x7fffffff;
      if (!lfu && key32) {
        // lexicographic (stamp, slot) minimum: the lane's own slots in
        // ascending order, then the minimum stamp and the lowest slot with it
        int key = INT32_MAX, bi = INT32_MAX;
        for (int c = lane; c < C; c += 32) {
          const int v = (int)s_stamp[c];
          if (v < key) { key = v; bi = c; }
        }
        const int m = __reduce_min_sync(full, key);
        best = __reduce_min_sync(full, key == m ? bi : INT32_MAX);
      } else if (!lfu) {
        int64_t key = INT64_MAX;
        for (int c = lane; c < C; c += 32)
          if (s_stamp[c] < key) { key = s_stamp[c]; best = c; }
        warp_argmin(key, best);
      } else {
        int64_t bu = INT64_MAX, bf = INT64_MAX, bi = INT64_MAX;
        for (int c = lane; c < C; c += 32) {
          const int64_t u = s_stamp[c] == step ? 1 : 0, f = s_freq[c], n = s_ins[c];
          if (u < bu || (u == bu && (f < bf || (f == bf && (n < bi || (n == bi && c < best)))))) {
            bu = u; bf = f; bi = n; best = c;
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          const int64_t ou = __shfl_xor_sync(full, bu, off);
          const int64_t of = __shfl_xor_sync(full, bf, off);
          const int64_t on = __shfl_xor_sync(full, bi, off);
          const int oc = __shfl_xor_sync(full, best, off);
          if (ou < bu || (ou == bu && (of < bf || (of == bf && (on < bi || (on == bi && oc < best)))))) {
            bu = ou; bf = of; bi = on; best = oc;
          }
        }
      }
      if (lane == 0) {
        const int32_t victim = s_owner[best];
        if (victim >= 0) p.slot_of[victim] = -1;
        p.slot_of[e] = best;
        p.slot_expert[best] = e;
        s_owner[best] = e;
        p.fetch_slot[nmiss] = best;
        p.fetch_expert[nmiss] = e;
        if (lfu) {
          s_freq[best] = 0;
          s_ins[best] = (step << 8) | i;
        }
      }
      ++nmiss;
      s = best;
    } else {
      ++hits;
    }
    if (lane == 0) {
      s_stamp[s] = step;
      p.stamp[s] = step;
      if (lfu) {
        s_freq[s] += 1;
        p.freq[s] = s_freq[s];
        p.ins[s] = s_ins[s];
      }
      p.out_slot[i] = s;
    }
    if (i < 32) { if (lane == i) out_lo = s; } else { if (lane == i - 32) out_hi = s; }
    __syncwarp();  // lane 0's shared-memory updates are seen by the next id
  }
  if (lane == 0) {
    *p.step = step;
    *p.nmiss = nmiss;
    if (p.counters) {
      atomicAdd(reinterpret_cast<unsigned long long*>(p.counters + 0), 1ull);
      atomicAdd(reinterpret_cast<unsigned long long*>(p.counters + 1), (unsigned long long)hits);
      atomicAdd(reinterpret_cast<unsigned long long*>(p.counters + 2), (unsigned long long)nmiss);
      atomicAdd(reinterpret_cast<unsigned long long*>(p.counters + 3),
                (unsigned long long)(nmiss * p.expert_bytes));
    }
  }
}

// ---------------------------------------------------------------- prefill gather

// One CTA: which experts a batch routes to.  present[] bitmap in shared memory,
// a block scan turns it into the ascending expert list and the expert ->
// compact index map; every pair's id is rewritten to its compact index.
__global__ void __launch_bounds__(1024) prefill_plan_kernel(const void* ids, int ids_bytes,
                                                            int n_pairs, int E,
                                                            int32_t* __restrict__ list,
                                                            int32_t* __restrict__ n_distinct,
                                                            int32_t* __restrict__ remap,
                                                            int32_t* __restrict__ local_ids) {
  extern __shared__ int32_t s_present[];  // [E]
  __shared__ int s_warp[32];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += blockDim.x) s_present[e] = 0;
  __syncthreads();
  for (int i = tid; i < n_pairs; i += blockDim.x) {
    const int32_t e = load_id(ids, ids_bytes, i);
    if (e >= 0 && e < E) s_present[e] = 1;
  }
  __syncthreads();
  // exclusive scan of present[] over contiguous per-thread ranges
  const int per = (E + blockDim.x - 1) / blockDim.x;
  const int lo = tid * per, hi = min(E, lo + per);
  int cnt = 0;
  for (int e = lo; e < hi; ++e) cnt += s_present[e];
  int v = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += a;
  }
  if (lane == 31) s_warp[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int a = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int b = __shfl_up_sync(0xffffffffu, a, o);
      if (lane >= o) a += b;
    }
    s_warp[lane] = a;
  }
  __syncthreads();
  int pos = (v - cnt) + (warp > 0 ? s_warp[warp - 1] : 0);
  for (int e = lo; e < hi; ++e) {
    if (s_present[e]) {
      list[pos] = e;
      remap[e] = pos;
      s_present[e] = pos + 1;  // keep compact index (+1) for the id rewrite
      ++pos;
    } else {
      remap[e] = -1;
    }
  }
  if (tid == 0) *n_distinct = s_warp[31];
  __syncthreads();
  for (int i = tid; i < n_pairs; i += blockDim.x) {
    const int32_t e = load_id(ids, ids_bytes, i);
    local_ids[i] = (e >= 0 && e < E) ? s_present[e] - 1 : -1;
  }
}

struct GatherParams {
  FetchParams f;                  // host/cache bases and per-buffer sizes (job fields unused)
  uint4* dst[D3_MAX_BUFFERS];     // compact buffers [n_max][bytes[b]]
  const int32_t* list;            // experts to gather, compact order
  const int32_t* n_distinct;
  const int32_t* slot_of;         // device cache map (read only), or null
  int32_t num_experts;
  int64_t* counters;              // {borrowed from cache, fetched from host}, or null
};

// Flat copy over n_distinct experts x all buffers: a cached expert is read
// from its device slot (read-only borrow: no stamp, no insert), any other from
// mapped pinned host memory.
__global__ void __launch_bounds__(kFetchThreads) gather_kernel(GatherParams p) {
  pdl_trigger();
  pdl_wait();
  const int nd = *p.n_distinct;
  if (nd <= 0) return;
  if (blockIdx.x == 0 && threadIdx.x < 32 && p.counters) {
    int borrowed = 0;
    for (int j = threadIdx.x; j < nd; j += 32)
      borrowed += (p.slot_of && p.slot_of[p.list[j]] >= 0) ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) borrowed += __shfl_xor_sync(0xffffffffu, borrowed, o);
    if (threadIdx.x == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(p.counters + 0), (unsigned long long)borrowed);
      atomicAdd(reinterpret_cast<unsigned long long*>(p.counters + 1),
                (unsigned long long)(nd - borrowed));
    }
  }
  const FetchParams& f = p.f;
  const int64_t total = (int64_t)nd * f.vec_total;
  constexpr int64_t kChunk = (int64_t)kFetchThreads * kFetchUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kChunk; base < total;
       base += (int64_t)gridDim.x * kChunk) {
    uint4 v[kFetchUnroll];
    uint4* dptr[kFetchUnroll];
#pragma unroll
    for (int u = 0; u < kFetchUnroll; ++u) {
      const int64_t g = base + (int64_t)u * kFetchThreads + threadIdx.x;
      dptr[u] = nullptr;
      if (g < total) {
        const int64_t j = g / f.vec_total;
        int64_t r = g - j * f.vec_total;
        int b = 0;
        while (b < f.nbuf - 1 && r >= f.vecs[b]) { r -= f.vecs[b]; ++b; }
        const int64_t e = p.list[j];
        const int s = p.slot_of ? p.slot_of[e] : -1;
        if (s >= 0)
          v[u] = f.cache[b][(int64_t)s * f.vecs[b] + r];
        else
          v[u] = ld_stream_u4(f.host[b] + e * f.vecs[b] + r);
        dptr[u] = p.dst[b] + j * f.vecs[b] + r;
      }
    }
#pragma unroll
    for (int u = 0; u < kFetchUnroll; ++u)
      if (dptr[u]) *dptr[u] = v[u];
  }
}

__global__ void lookup_kernel(const int32_t* __restrict__ slot_of, int32_t E, const void* ids,
                              int32_t ids_bytes, int32_t n, int32_t* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t e = load_id(ids, ids_bytes, i);
  out[i] = (e >= 0 && e < E) ? slot_of[e] : -1;
}

// ---------------------------------------------------------------- host side

static int launch_resolve(ResolveParams p, cudaStream_t st) {
  size_t smem = (size_t)p.capacity * sizeof(int64_t) * (p.policy == D3_POLICY_LFU ? 3 : 1) +
                (size_t)p.capacity * sizeof(int32_t);
  // the whole slot_of table beside the slot tables while that stays small
  const size_t slot_of_bytes = (size_t)p.num_experts * sizeof(int32_t);
  p.slot_of_smem = smem + slot_of_bytes <= 64 * 1024 ? 1 : 0;
  if (p.slot_of_smem) smem += slot_of_bytes;
  smem += (size_t)p.capacity;   // the LRU fast path's per-slot marks
  if (smem > 48 * 1024) {
    D3_CUDA_TRY(cudaFuncSetAttribute(resolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem),
                "resolve smem attribute");
  }
  // programmatic launch: resolve reads nothing before griddepcontrol.wait
  D3_CUDA_TRY(launch_k(resolve_kernel, dim3(1), dim3(32), smem, st, pdl_enabled(), p),
              "resolve_kernel launch");
  return D3_OK;
}

static int make_fetch_params(const d3_layer_cache* L, FetchParams* fp, int64_t* expert_bytes) {
  *expert_bytes = 0;
  for (int b = 0; b < L->nbuf; ++b) {
    D3_CHECK_ARG(L->host[b] && L->cache[b], "buffer %d: null host or cache pointer", b);
    if (L->bytes[b] <= 0 || L->bytes[b] % 16)
      return fail(D3_ERR_MISALIGNED, "buffer %d: bytes per expert %lld not a multiple of 16", b,
                  (long long)L->bytes[b]);
    if (!aligned16(L->host[b]) || !aligned16(L->cache[b]))
      return fail(D3_ERR_MISALIGNED, "buffer %d: base pointer not 16 B aligned", b);
    fp->host[b] = static_cast<const uint4*>(L->host[b]);
    fp->cache[b] = static_cast<uint4*>(L->cache[b]);
    fp->vecs[b] = L->bytes[b] / 16;
    fp->vec_total += fp->vecs[b];
    *expert_bytes += L->bytes[b];
  }
  fp->nbuf = L->nbuf;
  fp->fetch_slot = L->fetch_slot;
  fp->fetch_expert = L->fetch_expert;
  fp->nmiss = L->nmiss;
  return D3_OK;
}

// One fetch launch; with `pdl` it may start before the preceding allocator
// launch finishes (its griddepcontrol.wait then blocks until that grid's
// writes are visible).
static int launch_fetch(const FetchParams& fp, int fetch_ctas, cudaStream_t st, bool pdl) {
  const int ctas = fetch_ctas > 0 ? fetch_ctas : num_sms();
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kFetchThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  D3_CUDA_TRY(cudaLaunchKernelEx(&cfg, fetch_layer_kernel, fp), "fetch_layer_kernel launch");
  return D3_OK;
}

int resolve_for_fetch(const d3_layer_cache* L, const void* ids, int32_t ids_bytes, int32_t k,
                      int64_t* zero, int32_t nzero, cudaStream_t st, FetchParams* fp,
                      int64_t* expert_bytes, bool launch) {
  D3_CHECK_ARG(L && ids, "d3_resolve_fetch: null pointer");
  D3_CHECK_ARG(ids_bytes == 4 || ids_bytes == 8, "ids_bytes must be 4 or 8");
  D3_CHECK_ARG(k >= 1 && k <= 64, "k must be in [1, 64] (got %d)", k);
  D3_CHECK_ARG(L->num_experts >= 1, "num_experts must be >= 1");
  if (L->capacity < 1 || L->capacity > 8192)
    return fail(D3_ERR_TOO_LARGE, "capacity must be in [1, 8192] (got %d)", L->capacity);
  D3_CHECK_ARG(L->policy == D3_POLICY_LRU || L->policy == D3_POLICY_LFU, "unknown policy %d",
               L->policy);
  D3_CHECK_ARG(L->nbuf >= 1 && L->nbuf <= D3_MAX_BUFFERS, "nbuf must be in [1, %d]",
               D3_MAX_BUFFERS);
  D3_CHECK_ARG(L->slot_of && L->slot_expert && L->stamp && L->step && L->out_slot &&
                   L->fetch_slot && L->fetch_expert && L->nmiss,
               "d3_resolve_fetch: null table pointer");
  if (L->policy == D3_POLICY_LFU)
    D3_CHECK_ARG(L->freq && L->ins, "LFU needs freq and ins tables");
  D3_CHECK_ARG(nzero >= 0 && nzero <= 64 && (nzero == 0 || zero), "zero list out of range");
  *fp = FetchParams{};
  int rc = make_fetch_params(L, fp, expert_bytes);
  if (rc) return rc;
  ResolveParams p{};
  p.ids = ids; p.ids_bytes = ids_bytes; p.k = k; p.num_experts = L->num_experts;
  p.capacity = L->capacity; p.policy = L->policy;
  p.slot_of = L->slot_of; p.slot_expert = L->slot_expert; p.stamp = L->stamp; p.step = L->step;
  p.freq = L->freq; p.ins = L->ins;
  p.out_slot = L->out_slot; p.fetch_slot = L->fetch_slot; p.fetch_expert = L->fetch_expert;
  p.nmiss = L->nmiss; p.counters = L->counters; p.expert_bytes = *expert_bytes;
  p.zero = zero; p.nzero = nzero;
  return launch ? launch_resolve(p, st) : D3_OK;
}

}  // namespace d3

using namespace d3;

extern "C" {

const char* d3_last_error(void) { return g_last_error; }

int d3_abi_version(void) { return 1; }

const char* d3_status_string(int status) {
  switch (status) {
    case D3_OK: return "D3_OK";
    case D3_ERR_INVALID_ARG: return "D3_ERR_INVALID_ARG";
    case D3_ERR_NOT_PINNED: return "D3_ERR_NOT_PINNED";
    case D3_ERR_MISALIGNED: return "D3_ERR_MISALIGNED";
    case D3_ERR_CUDA: return "D3_ERR_CUDA";
    case D3_ERR_UNSUPPORTED: return "D3_ERR_UNSUPPORTED";
    case D3_ERR_TOO_LARGE: return "D3_ERR_TOO_LARGE";
    case D3_ERR_WORKSPACE: return "D3_ERR_WORKSPACE";
    default: return "D3_ERR_UNKNOWN";
  }
}

int d3_device_ptr_of(const void* host, size_t bytes, void** dev_out) {
  D3_CHECK_ARG(host && dev_out, "d3_device_ptr_of: null pointer");
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, host);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(e, "cudaPointerGetAttributes");
  }
  if (attr.type != cudaMemoryTypeHost)
    return fail(D3_ERR_NOT_PINNED,
                "expected page-locked (pinned) host memory; pointer %p has memory type %d", host,
                (int)attr.type);
  void* dptr = nullptr;
  D3_CUDA_TRY(cudaHostGetDevicePointer(&dptr, const_cast<void*>(host), 0),
              "cudaHostGetDevicePointer");
  // the whole range must be page-locked and device-mapped contiguously (it
  // may span adjacent registrations, whose device addresses then continue)
  if (bytes > 1) {
    cudaPointerAttributes last;
    const char* end = static_cast<const char*>(host) + bytes - 1;
    e = cudaPointerGetAttributes(&last, end);
    void* dend = nullptr;
    if (e == cudaSuccess && last.type == cudaMemoryTypeHost)
      e = cudaHostGetDevicePointer(&dend, const_cast<char*>(end), 0);
    if (e != cudaSuccess || last.type != cudaMemoryTypeHost ||
        static_cast<char*>(dend) != static_cast<char*>(dptr) + bytes - 1) {
      cudaGetLastError();
      return fail(D3_ERR_NOT_PINNED,
                  "range [%p, +%zu) is not one contiguously mapped page-locked range", host,
                  bytes);
    }
  }
  *dev_out = dptr;
  return D3_OK;
}

int d3_fetch_experts(const void* src_dev_base, void* dst, const int32_t* idx, const int32_t* slot,
                     const int32_t* njobs, int64_t expert_bytes, int32_t max_jobs,
                     int32_t blocks_per_job, int32_t threads, d3_stream_t stream) {
  D3_CHECK_ARG(src_dev_base && dst && idx && slot && njobs, "d3_fetch_experts: null pointer");
  if (expert_bytes <= 0 || expert_bytes % 16)
    return fail(D3_ERR_MISALIGNED, "expert_bytes must be a positive multiple of 16 (got %lld)",
                (long long)expert_bytes);
  if (!aligned16(src_dev_base)) return fail(D3_ERR_MISALIGNED, "host base must be 16 B aligned");
  if (!aligned16(dst)) return fail(D3_ERR_MISALIGNED, "cache base must be 16 B aligned");
  D3_CHECK_ARG(threads == 256, "threads must be 256 (kernel built with __launch_bounds__(256))");
  D3_CHECK_ARG(max_jobs >= 1 && max_jobs <= 65535, "max_jobs out of range");
  D3_CHECK_ARG(blocks_per_job >= 1 && blocks_per_job <= 65535, "blocks_per_job out of range");
  if (max_jobs == 0) return D3_OK;
  const dim3 grid((unsigned)blocks_per_job, (unsigned)max_jobs);
  fetch_jobs_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      static_cast<const uint4*>(src_dev_base), static_cast<uint4*>(dst), idx, slot, njobs,
      expert_bytes / 16);
  return launch_status("fetch_jobs_kernel launch");
}

int d3_resolve_slots(const void* ids, int32_t ids_bytes, int32_t k, int32_t* slot_of,
                     int32_t num_experts, int32_t* slot_expert, int64_t* stamp, int32_t capacity,
                     int32_t* out_slot, int32_t* fetch_slot, int32_t* fetch_expert, int32_t* nmiss,
                     int64_t* step, d3_stream_t stream) {
  D3_CHECK_ARG(ids && slot_of && slot_expert && stamp && out_slot && fetch_slot && fetch_expert &&
                   nmiss && step,
               "d3_resolve_slots: null pointer");
  D3_CHECK_ARG(ids_bytes == 4 || ids_bytes == 8, "ids_bytes must be 4 or 8");
  D3_CHECK_ARG(k >= 1 && k <= 64, "k must be in [1, 64] (got %d)", k);
  D3_CHECK_ARG(num_experts >= 1, "num_experts must be >= 1");
  if (capacity < 1 || capacity > 8192)
    return fail(D3_ERR_TOO_LARGE, "capacity must be in [1, 8192] (got %d)", capacity);
  ResolveParams p{};
  p.ids = ids; p.ids_bytes = ids_bytes; p.k = k; p.num_experts = num_experts;
  p.capacity = capacity; p.policy = D3_POLICY_LRU;
  p.slot_of = slot_of; p.slot_expert = slot_expert; p.stamp = stamp; p.step = step;
  p.out_slot = out_slot; p.fetch_slot = fetch_slot; p.fetch_expert = fetch_expert;
  p.nmiss = nmiss;
  return launch_resolve(p, (cudaStream_t)stream);
}

int d3_resolve_fetch(const d3_layer_cache* L, const void* ids, int32_t ids_bytes, int32_t k,
                     int32_t fetch_ctas, d3_stream_t stream) {
  D3_CHECK_ARG(fetch_ctas >= 0 && fetch_ctas <= 65535, "fetch_ctas out of range");
  FetchParams fp{};
  int64_t expert_bytes = 0;
  cudaStream_t st = (cudaStream_t)stream;
  const int rc = resolve_for_fetch(L, ids, ids_bytes, k, nullptr, 0, st, &fp, &expert_bytes);
  if (rc) return rc;
  return launch_fetch(fp, fetch_ctas, st, pdl_enabled());
}

int d3_fetch_jobs(const d3_layer_cache* L, int32_t fetch_ctas, d3_stream_t stream) {
  D3_CHECK_ARG(L, "d3_fetch_jobs: null descriptor");
  D3_CHECK_ARG(L->nbuf >= 1 && L->nbuf <= D3_MAX_BUFFERS, "nbuf must be in [1, %d]",
               D3_MAX_BUFFERS);
  D3_CHECK_ARG(L->fetch_slot && L->fetch_expert && L->nmiss, "d3_fetch_jobs: null job table");
  D3_CHECK_ARG(fetch_ctas >= 0 && fetch_ctas <= 65535, "fetch_ctas out of range");
  FetchParams fp{};
  int64_t expert_bytes = 0;
  int rc = make_fetch_params(L, &fp, &expert_bytes);
  if (rc) return rc;
  return launch_fetch(fp, fetch_ctas, (cudaStream_t)stream, false);
}

int d3_prefill_plan(const void* ids, int32_t ids_bytes, int32_t n_pairs, int32_t num_experts,
                    int32_t* expert_list, int32_t* n_distinct, int32_t* remap, int32_t* local_ids,
                    d3_stream_t stream) {
  D3_CHECK_ARG(ids && expert_list && n_distinct && remap && local_ids,
               "d3_prefill_plan: null pointer");
  D3_CHECK_ARG(ids_bytes == 4 || ids_bytes == 8, "ids_bytes must be 4 or 8");
  D3_CHECK_ARG(n_pairs >= 1, "n_pairs must be >= 1");
  if (num_experts < 1 || num_experts > 16384)
    return fail(D3_ERR_TOO_LARGE, "num_experts must be in [1, 16384]");
  const size_t smem = sizeof(int32_t) * (size_t)num_experts;
  if (smem > 48 * 1024)
    D3_CUDA_TRY(cudaFuncSetAttribute(prefill_plan_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "prefill plan smem attribute");
  D3_CUDA_TRY(launch_k(prefill_plan_kernel, dim3(1), dim3(1024), smem, (cudaStream_t)stream,
                       false, ids, ids_bytes, n_pairs, num_experts, expert_list,
                       n_distinct, remap, local_ids),
              "prefill_plan_kernel launch");
  return D3_OK;
}

int d3_gather_experts(const d3_layer_cache* L, const int32_t* expert_list,
                      const int32_t* n_distinct, void* const* dst, int64_t* counters,
                      int32_t fetch_ctas, d3_stream_t stream) {
  D3_CHECK_ARG(L && expert_list && n_distinct && dst, "d3_gather_experts: null pointer");
  D3_CHECK_ARG(L->nbuf >= 1 && L->nbuf <= D3_MAX_BUFFERS, "nbuf must be in [1, %d]",
               D3_MAX_BUFFERS);
  D3_CHECK_ARG(fetch_ctas >= 0 && fetch_ctas <= 65535, "fetch_ctas out of range");
  GatherParams gp{};
  int64_t expert_bytes = 0;
  // a layer without a device cache may pass null cache pointers: nothing is borrowed
  for (int b = 0; b < L->nbuf; ++b) {
    D3_CHECK_ARG(L->host[b] && dst[b], "buffer %d: null host or destination pointer", b);
    if (L->bytes[b] <= 0 || L->bytes[b] % 16)
      return fail(D3_ERR_MISALIGNED, "buffer %d: bytes per expert %lld not a multiple of 16", b,
                  (long long)L->bytes[b]);
    if (!aligned16(L->host[b]) || !aligned16(dst[b]) || (L->cache[b] && !aligned16(L->cache[b])))
      return fail(D3_ERR_MISALIGNED, "buffer %d: base pointer not 16 B aligned", b);
    if (L->slot_of) D3_CHECK_ARG(L->cache[b], "buffer %d: slot_of given without a cache", b);
    gp.f.host[b] = static_cast<const uint4*>(L->host[b]);
    gp.f.cache[b] = static_cast<uint4*>(L->cache[b]);
    gp.f.vecs[b] = L->bytes[b] / 16;
    gp.f.vec_total += gp.f.vecs[b];
    gp.dst[b] = static_cast<uint4*>(dst[b]);
    expert_bytes += L->bytes[b];
  }
  gp.f.nbuf = L->nbuf;
  gp.list = expert_list;
  gp.n_distinct = n_distinct;
  gp.slot_of = L->slot_of;
  gp.num_experts = L->num_experts;
  gp.counters = counters;
  const int ctas = fetch_ctas > 0 ? fetch_ctas : num_sms();
  D3_CUDA_TRY(launch_k(gather_kernel, dim3((unsigned)ctas), dim3(kFetchThreads), 0,
                       (cudaStream_t)stream, false, gp),
              "gather_kernel launch");
  return D3_OK;
}

int d3_lookup_slots(const int32_t* slot_of, int32_t num_experts, const void* ids,
                    int32_t ids_bytes, int32_t n, int32_t* slot_out, d3_stream_t stream) {
  D3_CHECK_ARG(slot_of && ids && slot_out, "d3_lookup_slots: null pointer");
  D3_CHECK_ARG(ids_bytes == 4 || ids_bytes == 8, "ids_bytes must be 4 or 8");
  D3_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return D3_OK;
  lookup_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(slot_of, num_experts, ids,
                                                                    ids_bytes, n, slot_out);
  return launch_status("lookup_kernel launch");
}

}  // extern "C"
