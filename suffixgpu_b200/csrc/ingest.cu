// Document ingestion into the global index's buffers: the device side of
// GlobalIndex.append_documents and of the delta's compaction
// (reference: suffix_gpu/global_index.py:86-133, 191-199; there each
// document is one slice copy plus a one-element SEP write plus a device
// length fill, and the compaction is a clone and a copy).
//
// sg_append_documents writes a whole batch of documents, each followed by
// SEP, in one launch per 32 documents; sg_delta_compact moves the delta's
// surviving tail to its front in one launch. Both set the device length
// scalar the delta queries read, so the host never touches it separately.
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

constexpr int kDocsPerLaunch = 32;
constexpr int kIngestThreads = 256;
constexpr int kSepToken = -2;

// One launch's documents, passed by value in the kernel parameters.
struct DocBatch {
  const int32_t* src[kDocsPerLaunch];
  int64_t dst[kDocsPerLaunch];  // offset of the document's first token
  int32_t len[kDocsPerLaunch];
  int32_t n;
};

// blockIdx.y = document; blockIdx.x strides over its tokens. The token
// that follows a document is SEP. The last launch of a call also writes
// the buffer's new length.
__global__ void __launch_bounds__(kIngestThreads)
    append_docs_kernel(int32_t* buf, const DocBatch batch, int64_t* len_out,
                       int64_t new_len) {
  const int d = blockIdx.y;
  if (d >= batch.n) return;
  const int32_t* src = batch.src[d];
  int32_t* dst = buf + batch.dst[d];
  const int n = batch.len[d];
  const int stride = gridDim.x * kIngestThreads;
  for (int i = blockIdx.x * kIngestThreads + threadIdx.x; i < n; i += stride)
    dst[i] = src[i];
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    dst[n] = kSepToken;
    if (d == 0 && len_out) *len_out = new_len;
  }
}

// Moves buf[from, from + count) to buf[0, count) with one block walking the
// range front to back, one tile per step: a tile's reads all happen before
// its writes (the barrier between them), and a write at position i < from
// + i never reaches a later tile's source, so the overlapping move is
// exact. Then *len_out = count.
constexpr int kCompactThreads = 1024;
constexpr int kCompactPerThread = 8;

__global__ void __launch_bounds__(kCompactThreads)
    delta_compact_kernel(int32_t* buf, int64_t from, int64_t count,
                         int64_t* len_out) {
  constexpr int kTile = kCompactThreads * kCompactPerThread;
  for (int64_t base = 0; base < count; base += kTile) {
    int32_t v[kCompactPerThread];
#pragma unroll
    for (int j = 0; j < kCompactPerThread; ++j) {
      const int64_t i = base + j * kCompactThreads + threadIdx.x;
      v[j] = i < count ? buf[from + i] : 0;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kCompactPerThread; ++j) {
      const int64_t i = base + j * kCompactThreads + threadIdx.x;
      if (i < count) buf[i] = v[j];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && len_out) *len_out = count;
}

__global__ void set_i64_kernel(int64_t* p, int64_t v) { *p = v; }

}  // namespace sg

using namespace sg;

extern "C" int sg_append_documents(int32_t* buf, int64_t capacity,
                                   int64_t start, const int32_t* const* docs,
                                   const int64_t* lens, int32_t n_docs,
                                   int64_t* len_out, sg_stream_t stream) {
  sg::NvtxScope nvtx_range("sg_append_documents");
  if (!buf || capacity < 0 || start < 0 || start > capacity || n_docs < 0 ||
      (n_docs > 0 && (!docs || !lens)))
    return SG_ERR_INVALID;
  int64_t end = start;
  int32_t longest = 0;
  for (int32_t i = 0; i < n_docs; ++i) {
    if (lens[i] < 0 || lens[i] > INT32_MAX - 1 || (lens[i] > 0 && !docs[i]))
      return SG_ERR_INVALID;
    end += lens[i] + 1;
    if (end > capacity) return SG_ERR_INVALID;  // nothing launched
    if (lens[i] > longest) longest = static_cast<int32_t>(lens[i]);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (n_docs == 0) {
    if (len_out) set_i64_kernel<<<1, 1, 0, st>>>(len_out, start);
    return check_launch();
  }
  const int64_t per_block = static_cast<int64_t>(kIngestThreads) * 4;
  const unsigned gx = static_cast<unsigned>(
      ceil_div(longest > 0 ? longest : 1, per_block) < 64
          ? ceil_div(longest > 0 ? longest : 1, per_block)
          : 64);
  int64_t pos = start;
  for (int32_t first = 0; first < n_docs; first += kDocsPerLaunch) {
    DocBatch b{};
    b.n = n_docs - first < kDocsPerLaunch ? n_docs - first : kDocsPerLaunch;
    for (int j = 0; j < b.n; ++j) {
      b.src[j] = docs[first + j];
      b.len[j] = static_cast<int32_t>(lens[first + j]);
      b.dst[j] = pos;
      pos += lens[first + j] + 1;
    }
    const bool last = first + kDocsPerLaunch >= n_docs;
    append_docs_kernel<<<dim3(gx, static_cast<unsigned>(b.n)),
                         kIngestThreads, 0, st>>>(
        buf, b, last ? len_out : nullptr, end);
  }
  return check_launch();
}

extern "C" int sg_delta_compact(int32_t* buf, int64_t capacity, int64_t from,
                                int64_t count, int64_t* len_out,
                                sg_stream_t stream) {
  if (!buf || from < 0 || count < 0 || from + count > capacity)
    return SG_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (from == 0 || count == 0) {
    if (len_out) set_i64_kernel<<<1, 1, 0, st>>>(len_out, count);
    return check_launch();
  }
  delta_compact_kernel<<<1, kCompactThreads, 0, st>>>(buf, from, count,
                                                      len_out);
  return check_launch();
}
