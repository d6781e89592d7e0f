// Routing observability on the device: the [layer, expert] census and the
// router trace.
//
// The reference keeps both on the host (bin/offload.py:40-79 RouterTrace,
// :257-287 enable_census/_count): every MoE call copies its top-k ids to the
// CPU (a device sync per layer) and bincounts or appends them.  Here both are
// device launches on the caller's stream -- no sync, graph-capturable -- and
// the host reads the buffers only when it asks for them.
//
//   census   counts[e] += occurrences of e among the call's ids; a call of
//            exactly one row (a decode step) also adds to the decode census.
//            Out-of-range ids are not counted.
//   trace    every row of the call appends one record to a ring of
//            `capacity` records: {first row of the call, layer, phase
//            (0 prefill / 1 decode), ids[k]}; the 64-bit cursor counts all
//            rows ever appended, so the host knows what wrapped.
#include "d3_common.cuh"

namespace d3 {

__device__ __forceinline__ long long census_load_id(const void* ids, int bytes, int i) {
  return bytes == 8 ? static_cast<const long long*>(ids)[i]
                    : (long long)static_cast<const int*>(ids)[i];
}

__global__ void census_kernel(const void* ids, int ids_bytes, int n_ids, int num_experts,
                              unsigned long long* counts, unsigned long long* counts_decode) {
  pdl_trigger();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_ids; i += gridDim.x * blockDim.x) {
    const long long e = census_load_id(ids, ids_bytes, i);
    if (e < 0 || e >= num_experts) continue;
    atomicAdd(counts + e, 1ull);
    if (counts_decode) atomicAdd(counts_decode + e, 1ull);
  }
}

// One CTA: claims `rows` records with one atomic, then writes them.
__global__ void trace_kernel(const void* ids, int ids_bytes, int rows, int k, int layer,
                             int phase, int32_t* ring, unsigned long long* cursor,
                             long long capacity) {
  __shared__ unsigned long long s_base;
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) s_base = atomicAdd(cursor, (unsigned long long)rows);
  __syncthreads();
  const unsigned long long base = s_base;
  const int rec = 3 + k;
  for (int i = threadIdx.x; i < rows * rec; i += blockDim.x) {
    const int r = i / rec, f = i - r * rec;
    const unsigned long long slot = (base + (unsigned long long)r) % (unsigned long long)capacity;
    int32_t v;
    if (f == 0) v = (int32_t)(base & 0x7fffffffull);
    else if (f == 1) v = layer;
    else if (f == 2) v = phase;
    else v = (int32_t)census_load_id(ids, ids_bytes, r * k + (f - 3));
    ring[slot * rec + f] = v;
  }
}

}  // namespace d3

using namespace d3;

extern "C" {

int d3_census_add(const void* ids, int32_t ids_bytes, int32_t rows, int32_t k,
                  int32_t num_experts, int64_t* counts, int64_t* counts_decode,
                  d3_stream_t stream) {
  D3_CHECK_ARG(ids && counts, "d3_census_add: null pointer");
  D3_CHECK_ARG(ids_bytes == 4 || ids_bytes == 8, "ids_bytes must be 4 or 8");
  D3_CHECK_ARG(rows >= 1 && k >= 1 && (long)rows * k <= (1L << 30), "rows, k out of range");
  D3_CHECK_ARG(num_experts >= 1, "num_experts must be >= 1");
  const int n = rows * k;
  const unsigned blocks = (unsigned)((n + 255) / 256 < 148 ? (n + 255) / 256 : 148);
  D3_CUDA_TRY(launch_k(census_kernel, dim3(blocks), dim3(256), 0, (cudaStream_t)stream, false,
                       ids, (int)ids_bytes, n, (int)num_experts,
                       reinterpret_cast<unsigned long long*>(counts),
                       reinterpret_cast<unsigned long long*>(rows == 1 ? counts_decode : nullptr)),
              "census_kernel launch");
  return D3_OK;
}

int d3_trace_append(const void* ids, int32_t ids_bytes, int32_t rows, int32_t k, int32_t layer,
                    int32_t* ring, int64_t* cursor, int64_t capacity, d3_stream_t stream) {
  D3_CHECK_ARG(ids && ring && cursor, "d3_trace_append: null pointer");
  D3_CHECK_ARG(ids_bytes == 4 || ids_bytes == 8, "ids_bytes must be 4 or 8");
  D3_CHECK_ARG(rows >= 1 && k >= 1 && k <= 1024, "rows, k out of range");
  D3_CHECK_ARG(capacity >= 1, "capacity must be >= 1");
  if ((long long)rows > capacity)
    return fail(D3_ERR_TOO_LARGE, "a call of %d rows does not fit a ring of %lld records", rows,
                (long long)capacity);
  D3_CUDA_TRY(launch_k(trace_kernel, dim3(1), dim3(256), 0, (cudaStream_t)stream, false, ids,
                       (int)ids_bytes, (int)rows, (int)k, (int)layer, rows == 1 ? 1 : 0, ring,
                       reinterpret_cast<unsigned long long*>(cursor), (long long)capacity),
              "trace_kernel launch");
  return D3_OK;
}

}  // extern "C"
