// Input pipeline: Spar's LM batch iterator (data::LMBatchIterator, src/data/batch_iterator.cpp:
// 56-143) over the windows of a packed token corpus (data::WindowDataset, src/data/
// tokenized_corpus.cpp:49-80), with the corpus resident in HBM.
//
// Reference semantics, restated: window i is tokens [i * stride, i * stride + T); an epoch visits
// the windows in the order iota(window_count), Fisher-Yates shuffled (when shuffle is on) by a
// SplitMix64 Random seeded with derive_epoch_seed(shuffle_seed, epoch) (one SplitMix64 output of
// seed + golden * (epoch + 1)), each swap index drawn by bounded_index (reject draws below
// (2^64 - bound) % bound, then value % bound); batches take `batch_size` consecutive windows of
// that order (the last one shorter unless drop_last drops it); the state is (epoch, cursor).
//
// B200 side: the order lives on the host (it is O(windows) once per epoch); each batch sends only
// its window start offsets (rows x 8 bytes) to the device, where one kernel gathers the [rows, T]
// int32 token ids out of the resident corpus straight into the step's input buffer. For data
// parallelism each rank takes its contiguous share of every global batch (rows r * n / world ..
// (r + 1) * n / world), the split the benchmark's synthetic batches use.
#include <cuda_runtime.h>

#include <cstring>
#include <numeric>
#include <vector>

#include "common.cuh"

namespace spar_b200 {
namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t derive_epoch_seed(uint64_t seed, uint64_t epoch) { return mix64(seed + kGolden * (epoch + 1)); }

struct SplitMix {  // Spar's Random (src/core/random.cpp:22-28)
  uint64_t state;
  uint64_t next() {
    state += kGolden;
    return mix64(state);
  }
};

uint64_t bounded_index(SplitMix& r, uint64_t bound) {
  const uint64_t threshold = (0 - bound) % bound;
  uint64_t v;
  do {
    v = r.next();
  } while (v < threshold);
  return v % bound;
}

// Fisher-Yates over iota(n) with a Random seeded `seed` (batch_iterator.cpp:34-40).
void shuffled(std::vector<uint64_t>& order, uint64_t n, uint64_t seed) {
  order.resize(n);
  std::iota(order.begin(), order.end(), uint64_t{0});
  SplitMix r{seed};
  for (uint64_t remaining = n; remaining > 1; --remaining)
    std::swap(order[remaining - 1], order[bounded_index(r, remaining)]);
}

void epoch_order(std::vector<uint64_t>& order, uint64_t windows, bool shuffle, uint64_t seed,
                 uint64_t epoch) {
  if (shuffle) {
    shuffled(order, windows, derive_epoch_seed(seed, epoch));
    return;
  }
  order.resize(windows);
  std::iota(order.begin(), order.end(), uint64_t{0});
}

// This rank's rows of the batch starting at `cursor`: window starts into `starts`; returns the
// global batch size (0: epoch finished) and this rank's [row0, row1).
uint64_t next_rows(const std::vector<uint64_t>& order, uint64_t cursor, uint64_t batch,
                   bool drop_last, int rank, int world, uint64_t& row0, uint64_t& row1) {
  const uint64_t n = order.size();
  row0 = row1 = 0;
  if (cursor >= n) return 0;
  const uint64_t remaining = n - cursor;
  if (drop_last && remaining < batch) return 0;
  const uint64_t rows = remaining < batch ? remaining : batch;
  row0 = rows * static_cast<uint64_t>(rank) / static_cast<uint64_t>(world);
  row1 = rows * static_cast<uint64_t>(rank + 1) / static_cast<uint64_t>(world);
  return rows;
}

// ids[r, t] = corpus[starts[r] + t]; grid-stride over rows x T.
__global__ void gather_windows_kernel(int32_t* __restrict__ ids, const int32_t* __restrict__ corpus,
                                      const uint64_t* __restrict__ starts, uint64_t rows,
                                      uint64_t seq) {
  pdl_begin();
  const uint64_t total = rows * seq;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const uint64_t r = i / seq;
    ids[i] = corpus[starts[r] + (i - r * seq)];
  }
}

struct Batches {
  int device = 0, rank = 0, world = 1;
  uint64_t tokens = 0, seq = 0, stride = 0, batch = 0, windows = 0, seed = 0;
  bool shuffle = true, drop_last = false;
  uint64_t epoch = 0, cursor = 0;
  std::vector<uint64_t> order;
  int32_t* corpus = nullptr;       // device
  uint64_t* starts_dev = nullptr;  // device [batch]
  uint64_t* starts_host = nullptr; // pinned [batch]
  cudaEvent_t copied = nullptr;    // the last starts copy has read starts_host
  ~Batches() {
    DeviceScope scope(device);
    if (copied) {
      cudaEventSynchronize(copied);
      cudaEventDestroy(copied);
    }
    cudaFree(corpus);
    cudaFree(starts_dev);
    cudaFreeHost(starts_host);
  }
};

}  // namespace
}  // namespace spar_b200

using namespace spar_b200;

// Creates the iterator; copies the packed corpus (int32 token ids) to `device`.
extern "C" SparCudaStatus spar_b200_batches_create(const int32_t* tokens, uint64_t token_count,
                                                   uint64_t sequence_length, uint64_t stride,
                                                   uint64_t batch_size, int shuffle,
                                                   uint64_t shuffle_seed, int drop_last, int rank,
                                                   int world, int device, void** handle) {
  // WindowDataset / LMBatchIterator argument checks (tokenized_corpus.cpp:51-56,
  // batch_iterator.cpp:59-61).
  if (!handle || (token_count && !tokens) || sequence_length < 2 || stride == 0 ||
      stride > sequence_length || batch_size == 0 || world < 1 || rank < 0 || rank >= world)
    return invalid();
  *handle = nullptr;
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  Batches* b = new Batches();
  b->device = device;
  b->rank = rank;
  b->world = world;
  b->tokens = token_count;
  b->seq = sequence_length;
  b->stride = stride;
  b->batch = batch_size;
  b->windows = token_count >= sequence_length ? 1 + (token_count - sequence_length) / stride : 0;
  b->shuffle = shuffle != 0;
  b->seed = shuffle_seed;
  b->drop_last = drop_last != 0;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&b->corpus), (token_count ? token_count : 1) * 4);
  if (e == cudaSuccess && token_count)
    e = cudaMemcpy(b->corpus, tokens, token_count * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&b->starts_dev), batch_size * 8);
  if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&b->starts_host), batch_size * 8);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b->copied, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    delete b;
    return runtime(e);
  }
  epoch_order(b->order, b->windows, b->shuffle, b->seed, 0);
  *handle = b;
  return ok();
}

// Gathers this rank's rows of the next batch into ids (device, [rows, sequence_length] int32,
// ordered on `stream`). *global_rows (optional) receives the whole batch's row count, 0 when the
// epoch is finished (call next_epoch); *rows alone is 0 also for a rank whose share of a short
// last batch is empty.
extern "C" SparCudaStatus spar_b200_batches_next(void* handle, int32_t* ids, uint64_t* rows,
                                                 uint64_t* global_rows, void* stream) {
  if (!handle || !rows) return invalid();
  Batches* b = static_cast<Batches*>(handle);
  DeviceScope scope(b->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  uint64_t r0, r1;
  const uint64_t n = next_rows(b->order, b->cursor, b->batch, b->drop_last, b->rank, b->world, r0, r1);
  if (global_rows) *global_rows = n;
  *rows = r1 - r0;
  if (n == 0) {
    b->cursor = b->order.size();
    return ok();
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (*rows) {
    if (!ids) return invalid();
    cudaError_t e = cudaEventSynchronize(b->copied);  // the previous copy has read starts_host
    for (uint64_t r = r0; r < r1 && e == cudaSuccess; ++r)
      b->starts_host[r - r0] = b->order[b->cursor + r] * b->stride;
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(b->starts_dev, b->starts_host, *rows * 8, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(b->copied, s);
    if (e == cudaSuccess)
      e = launch(gather_windows_kernel, dim3(grid_for(*rows * b->seq, 256, sm_count(b->device) * 4)),
                 dim3(256), 0, s, ids, static_cast<const int32_t*>(b->corpus),
                 static_cast<const uint64_t*>(b->starts_dev), *rows, b->seq);
    if (e != cudaSuccess) return runtime(e);
  }
  b->cursor += n;
  return ok();
}

extern "C" SparCudaStatus spar_b200_batches_next_epoch(void* handle) {
  if (!handle) return invalid();
  Batches* b = static_cast<Batches*>(handle);
  if (b->epoch == ~uint64_t{0}) return invalid();
  ++b->epoch;
  b->cursor = 0;
  epoch_order(b->order, b->windows, b->shuffle, b->seed, b->epoch);
  return ok();
}

// BatchIteratorState (batch_iterator.cppm): the epoch and the windows of its order consumed.
extern "C" SparCudaStatus spar_b200_batches_state(void* handle, uint64_t* epoch, uint64_t* cursor,
                                                  uint64_t* windows) {
  if (!handle) return invalid();
  const Batches* b = static_cast<const Batches*>(handle);
  if (epoch) *epoch = b->epoch;
  if (cursor) *cursor = b->cursor;
  if (windows) *windows = b->windows;
  return ok();
}

extern "C" SparCudaStatus spar_b200_batches_set_state(void* handle, uint64_t epoch,
                                                      uint64_t cursor) {
  if (!handle) return invalid();
  Batches* b = static_cast<Batches*>(handle);
  if (cursor > b->windows) return invalid();  // LMBatchIterator::set_state's check
  b->epoch = epoch;
  b->cursor = cursor;
  epoch_order(b->order, b->windows, b->shuffle, b->seed, epoch);
  return ok();
}

extern "C" void spar_b200_batches_destroy(void* handle) { delete static_cast<Batches*>(handle); }

// Host-only (no GPU): this rank's window start offsets of the batch at (epoch, cursor) and the
// cursor after it; *rows = this rank's rows, *global_rows = the batch's (0: epoch finished).
extern "C" SparCudaStatus spar_b200_batch_windows(uint64_t token_count, uint64_t sequence_length,
                                                  uint64_t stride, uint64_t batch_size, int shuffle,
                                                  uint64_t shuffle_seed, int drop_last,
                                                  uint64_t epoch, uint64_t cursor, int rank,
                                                  int world, uint64_t* starts, uint64_t* rows,
                                                  uint64_t* global_rows, uint64_t* next_cursor) {
  if (!rows || !global_rows || !next_cursor || sequence_length < 2 || stride == 0 ||
      stride > sequence_length || batch_size == 0 || world < 1 || rank < 0 || rank >= world)
    return invalid();
  const uint64_t windows =
      token_count >= sequence_length ? 1 + (token_count - sequence_length) / stride : 0;
  if (cursor > windows) return invalid();
  std::vector<uint64_t> order;
  epoch_order(order, windows, shuffle != 0, shuffle_seed, epoch);
  uint64_t r0, r1;
  *global_rows = next_rows(order, cursor, batch_size, drop_last != 0, rank, world, r0, r1);
  *rows = r1 - r0;
  if (*rows && !starts) return invalid();
  for (uint64_t r = r0; r < r1; ++r) starts[r - r0] = order[cursor + r] * stride;
  *next_cursor = *global_rows ? cursor + *global_rows : windows;
  return ok();
}

// data::split_documents (batch_iterator.cpp:144-162): the document indices shuffled by Random(seed);
// the first validation_count are the validation documents, the rest (in that order) the training
// ones. order: document_count entries. Host-only.
extern "C" SparCudaStatus spar_b200_split_documents(uint64_t document_count,
                                                    uint64_t validation_count, uint64_t seed,
                                                    uint64_t* order) {
  if (validation_count > document_count || (document_count && !order)) return invalid();
  std::vector<uint64_t> o;
  shuffled(o, document_count, seed);
  if (document_count) std::memcpy(order, o.data(), document_count * sizeof(uint64_t));
  return ok();
}
