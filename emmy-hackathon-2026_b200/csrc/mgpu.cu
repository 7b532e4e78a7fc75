// Multi-GPU driver of the C ABI (include/b200k.h, b2k_mgpu_*): one process
// per GPU, one NCCL communicator per process, one problem partitioned over
// the ranks.  The reference is single-GPU (its runner drives one device,
// tools/local_runner.py:246-342); every workload of its hot path splits into
// independent units (rows of A with B replicated, softmax rows, element
// ranges, attention heads), so the only collectives are the broadcast of B
// from rank 0 and the all-gather of the outputs.  Both run on a stream of
// the communicator's own and overlap the compute on the caller's stream:
// B goes out in column panels and panel p's GEMM waits only for panel p;
// output pieces are gathered while the next piece computes.
//
// NCCL is opened at run time (dlopen of libnccl.so.2), so the library loads
// and every single-GPU entry point works on hosts without it; in a process
// that already holds NCCL (PyTorch's), the loaded copy is reused.  The
// communicator is created non-blocking so that a rank that never joins ends
// b2k_mgpu_init with B2K_ETIMEOUT instead of a hang, and b2k_mgpu_sync bounds
// the wait for a step's collectives the same way (aborting the communicator).
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"

namespace {

struct NcclApi {
  bool loaded = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
};

NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char *e = dlerror();
      api.why = e ? e : "libnccl.so.2 not found";
      return;
    }
    auto sym = [&](const char *name) {
      void *p = dlsym(h, name);
      if (!p && api.why.empty()) api.why = std::string("libnccl lacks ") + name;
      return p;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.init_rank_config = reinterpret_cast<decltype(api.init_rank_config)>(sym("ncclCommInitRankConfig"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(sym("ncclCommGetAsyncError"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
    api.abort = reinterpret_cast<decltype(api.abort)>(sym("ncclCommAbort"));
    api.broadcast = reinterpret_cast<decltype(api.broadcast)>(sym("ncclBroadcast"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.loaded = api.why.empty();
  });
  return api;
}

constexpr int kMaxSplits = 16;  // panels / pieces per call

}  // namespace

struct b2k_mgpu {
  b2k_ctx *ctx = nullptr;
  int world = 1, rank = 0;
  ncclComm_t comm = nullptr;
  bool broken = false;  // aborted after an error or a timeout
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t start = nullptr, done = nullptr, mark = nullptr;
  cudaEvent_t ready[kMaxSplits] = {}, computed[kMaxSplits] = {};
  float *ws = nullptr;
  size_t ws_floats = 0;
};

namespace {

using b2k::fail;
using b2k::cuda_fail;

int nccl_fail(b2k_mgpu *mg, ncclResult_t r, const char *what) {
  return fail(mg->ctx, B2K_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "nccl error");
}

// A non-blocking communicator may answer ncclInProgress; wait (bounded) until
// the operation has been taken, as NCCL requires before the next call.
int settle(b2k_mgpu *mg, ncclResult_t r, const char *what, int64_t timeout_ms = 60000) {
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      nccl().abort(mg->comm);
      mg->broken = true;
      return fail(mg->ctx, B2K_ETIMEOUT, "%s: no progress within %lld ms (communicator aborted)", what,
                  (long long)timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(5));
    nccl().async_error(mg->comm, &r);
  }
  if (r != ncclSuccess) {
    mg->broken = true;
    return nccl_fail(mg, r, what);
  }
  return B2K_OK;
}

int reserve(b2k_mgpu *mg, size_t floats, cudaStream_t s) {
  if (floats <= mg->ws_floats) return B2K_OK;
  // the staging buffers may still be read by the previous call's work
  cudaError_t err = cudaStreamSynchronize(s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(mg->comm_stream);
  if (err != cudaSuccess) return cuda_fail(mg->ctx, err, "mgpu: sync before growing staging");
  if (mg->ws) cudaFree(mg->ws);
  mg->ws = nullptr;
  mg->ws_floats = 0;
  const size_t rounded = (floats + (size_t(1) << 19) - 1) & ~((size_t(1) << 19) - 1);
  err = cudaMalloc(&mg->ws, rounded * sizeof(float));
  if (err != cudaSuccess) {
    mg->ws = nullptr;
    return cuda_fail(mg->ctx, err, "mgpu: staging cudaMalloc");
  }
  mg->ws_floats = rounded;
  return B2K_OK;
}

struct Part {
  int64_t start, count;
};

// The rank's shard of `units`: every shard but the last a multiple of
// `align`, the last taking the remainder (mgpu.partition in Python).
Part part_of(int64_t units, int world, int rank, int64_t align) {
  const int64_t base = (units / world) / align * align;
  return {base * rank, rank < world - 1 ? base : units - base * (world - 1)};
}

int check_handle(b2k_mgpu *mg) {
  if (!mg) return B2K_EINVAL;
  if (mg->broken) return fail(mg->ctx, B2K_ENCCL, "mgpu: communicator was aborted after an earlier error");
  return b2k::make_current(mg->ctx);
}

// Begin a step: the communicator's stream waits for everything issued on
// the caller's stream so far (inputs, and the previous step's reads of the
// staging buffers).
int begin(b2k_mgpu *mg, cudaStream_t s) {
  cudaError_t err = cudaEventRecord(mg->start, s);
  if (err == cudaSuccess) err = cudaStreamWaitEvent(mg->comm_stream, mg->start, 0);
  return err == cudaSuccess ? B2K_OK : cuda_fail(mg->ctx, err, "mgpu: order the step");
}

// End a step: the caller's stream waits for the gathers and copies.
int finish(b2k_mgpu *mg, cudaStream_t s) {
  cudaError_t err = cudaEventRecord(mg->done, mg->comm_stream);
  if (err == cudaSuccess) err = cudaStreamWaitEvent(s, mg->done, 0);
  return err == cudaSuccess ? B2K_OK : cuda_fail(mg->ctx, err, "mgpu: join the step");
}

int cuda_ok(b2k_mgpu *mg, cudaError_t err, const char *what) {
  return err == cudaSuccess ? B2K_OK : cuda_fail(mg->ctx, err, what);
}

// Gather a row-slab operation's output.  Rank r computed rows
// [start_r, start_r + count_r) of `out` (row_elems floats per row) in
// `pieces` pieces; piece i of every rank is gathered after event
// computed[i], on the communicator's stream.  Equal shards in one piece are
// gathered in place; otherwise through staging (padded to the largest shard
// for uneven ones) and copied to their rows.
int gather_rows(b2k_mgpu *mg, float *out, int64_t units, int64_t align, int64_t row_elems, int pieces,
                float *staging) {
  const int world = mg->world;
  std::vector<Part> parts(world);
  int64_t width = 0;
  bool equal = true;
  for (int r = 0; r < world; ++r) {
    parts[r] = part_of(units, world, r, align);
    width = std::max(width, parts[r].count);
    equal = equal && parts[r].count == parts[0].count;
  }
  if (width == 0) return B2K_OK;
  const Part mine = parts[mg->rank];
  const int64_t step = width / pieces;
  for (int i = 0; i < pieces; ++i) {
    int rc = cuda_ok(mg, cudaStreamWaitEvent(mg->comm_stream, mg->computed[i], 0), "mgpu: wait piece");
    if (rc) return rc;
    const size_t piece_floats = (size_t)(step * row_elems);
    if (equal && pieces == 1) {
      rc = settle(mg, nccl().all_gather(out + mine.start * row_elems, out, piece_floats, ncclFloat32, mg->comm,
                                        mg->comm_stream), "ncclAllGather");
      if (rc) return rc;
      continue;
    }
    float *send = out + (mine.start + i * step) * row_elems;
    float *recv = staging + (size_t)i * world * piece_floats;
    if (!equal) {
      // pad this rank's slab to the common width (the pad rows are never read)
      float *pad = staging + (size_t)world * width * row_elems;
      if (mine.count > 0) {
        rc = cuda_ok(mg, cudaMemcpyAsync(pad, send, (size_t)(mine.count * row_elems) * sizeof(float),
                                         cudaMemcpyDeviceToDevice, mg->comm_stream), "mgpu: pad slab");
        if (rc) return rc;
      }
      send = pad;
    }
    rc = settle(mg, nccl().all_gather(send, recv, piece_floats, ncclFloat32, mg->comm, mg->comm_stream),
                "ncclAllGather");
    if (rc) return rc;
    for (int r = 0; r < world; ++r) {
      if (r == mg->rank) continue;
      const int64_t rows = equal ? step : parts[r].count;
      if (rows == 0) continue;
      const int64_t at = parts[r].start + (equal ? i * step : 0);
      rc = cuda_ok(mg, cudaMemcpyAsync(out + at * row_elems, recv + (size_t)r * piece_floats,
                                       (size_t)(rows * row_elems) * sizeof(float), cudaMemcpyDeviceToDevice,
                                       mg->comm_stream), "mgpu: place gathered rows");
      if (rc) return rc;
    }
  }
  return B2K_OK;
}

// Pieces a row-slab step can use: equal shards cut into equal pieces of a
// multiple of `align` units; otherwise one.
int usable_pieces(int64_t units, int world, int64_t align, int pieces) {
  if (pieces <= 1) return 1;
  for (int r = 1; r < world; ++r)
    if (part_of(units, world, r, align).count != part_of(units, world, 0, align).count) return 1;
  const int64_t count = part_of(units, world, 0, align).count;
  if (count % pieces || (count / pieces) % align) return 1;
  return pieces;
}

// A row-slab operation: compute(start, count) writes rows [start, start +
// count) of this rank's slab (relative to the slab) into out at its rows.
template <class Compute>
int run_slabs(b2k_mgpu *mg, float *out, int64_t units, int64_t align, int64_t row_elems, int pieces,
              cudaStream_t s, Compute compute) {
  if (pieces < 1 || pieces > kMaxSplits) return fail(mg->ctx, B2K_EINVAL, "mgpu: pieces must be in 1..%d", kMaxSplits);
  pieces = usable_pieces(units, mg->world, align, pieces);
  const Part mine = part_of(units, mg->world, mg->rank, align);
  int64_t width = 0;
  for (int r = 0; r < mg->world; ++r) width = std::max(width, part_of(units, mg->world, r, align).count);
  int rc = reserve(mg, (size_t)((mg->world + 1) * width * row_elems), s);
  if (rc) return rc;
  rc = begin(mg, s);
  if (rc) return rc;
  const int64_t step = mine.count / pieces;
  for (int i = 0; i < pieces; ++i) {
    if (step > 0) {
      rc = compute(i * step, step);
      if (rc) return rc;
    }
    rc = cuda_ok(mg, cudaEventRecord(mg->computed[i], s), "mgpu: record piece");
    if (rc) return rc;
  }
  rc = gather_rows(mg, out, units, align, row_elems, pieces, mg->ws);
  if (rc) return rc;
  return finish(mg, s);
}

}  // namespace

extern "C" {

int b2k_mgpu_partition(int64_t units, int32_t world, int32_t rank, int64_t align, int64_t *start, int64_t *count) {
  if (units < 0 || world <= 0 || rank < 0 || rank >= world || align <= 0 || !start || !count) return B2K_EINVAL;
  const Part p = part_of(units, world, rank, align);
  *start = p.start;
  *count = p.count;
  return B2K_OK;
}

int b2k_mgpu_unique_id(void *id) {
  if (!id) return B2K_EINVAL;
  if (!nccl().loaded) return B2K_EUNSUPPORTED;
  ncclUniqueId uid;
  if (nccl().get_unique_id(&uid) != ncclSuccess) return B2K_ENCCL;
  memcpy(id, &uid, sizeof uid);
  return B2K_OK;
}

int b2k_mgpu_init(b2k_ctx *ctx, int32_t world, int32_t rank, const void *id, int64_t timeout_ms, b2k_mgpu **out) {
  static_assert(sizeof(ncclUniqueId) == B2K_MGPU_ID_BYTES, "NCCL unique id size");
  if (!ctx || !out || !id || world <= 0 || rank < 0 || rank >= world || timeout_ms <= 0) return B2K_EINVAL;
  *out = nullptr;
  if (!nccl().loaded) return fail(ctx, B2K_EUNSUPPORTED, "mgpu: NCCL unavailable (%s)", nccl().why.c_str());
  int rc = b2k::make_current(ctx);
  if (rc) return rc;
  auto *mg = new (std::nothrow) b2k_mgpu;
  if (!mg) return fail(ctx, B2K_ECUDA, "mgpu: out of host memory");
  mg->ctx = ctx;
  mg->world = world;
  mg->rank = rank;
  cudaError_t err = cudaStreamCreateWithFlags(&mg->comm_stream, cudaStreamNonBlocking);
  if (err == cudaSuccess) err = cudaEventCreateWithFlags(&mg->start, cudaEventDisableTiming);
  if (err == cudaSuccess) err = cudaEventCreateWithFlags(&mg->done, cudaEventDisableTiming);
  if (err == cudaSuccess) err = cudaEventCreateWithFlags(&mg->mark, cudaEventDisableTiming);
  for (int i = 0; i < kMaxSplits && err == cudaSuccess; ++i) {
    err = cudaEventCreateWithFlags(&mg->ready[i], cudaEventDisableTiming);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&mg->computed[i], cudaEventDisableTiming);
  }
  if (err != cudaSuccess) {
    b2k_mgpu_destroy(mg);
    return cuda_fail(ctx, err, "mgpu: streams and events");
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclResult_t r = nccl().init_rank_config(&mg->comm, world, uid, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) {
    rc = nccl_fail(mg, r, "ncclCommInitRankConfig");
    mg->comm = nullptr;
    b2k_mgpu_destroy(mg);
    return rc;
  }
  rc = settle(mg, r, "ncclCommInitRankConfig (waiting for every rank to join)", timeout_ms);
  if (rc) {
    b2k_mgpu_destroy(mg);
    return rc;
  }
  *out = mg;
  ctx->error.clear();
  return B2K_OK;
}

int b2k_mgpu_destroy(b2k_mgpu *mg) {
  if (!mg) return B2K_OK;
  if (mg->ctx) cudaSetDevice(mg->ctx->device);
  if (mg->comm_stream) cudaStreamSynchronize(mg->comm_stream);
  if (mg->comm) {
    if (mg->broken) {
      nccl().abort(mg->comm);
    } else {
      ncclResult_t r = nccl().destroy(mg->comm);
      if (r == ncclInProgress) settle(mg, r, "ncclCommDestroy", 10000);
    }
  }
  if (mg->ws) cudaFree(mg->ws);
  for (int i = 0; i < kMaxSplits; ++i) {
    if (mg->ready[i]) cudaEventDestroy(mg->ready[i]);
    if (mg->computed[i]) cudaEventDestroy(mg->computed[i]);
  }
  if (mg->start) cudaEventDestroy(mg->start);
  if (mg->done) cudaEventDestroy(mg->done);
  if (mg->mark) cudaEventDestroy(mg->mark);
  if (mg->comm_stream) cudaStreamDestroy(mg->comm_stream);
  delete mg;
  return B2K_OK;
}

int b2k_mgpu_sync(b2k_mgpu *mg, void *stream, int64_t timeout_ms) {
  int rc = check_handle(mg);
  if (rc) return rc;
  if (timeout_ms <= 0) return fail(mg->ctx, B2K_EINVAL, "mgpu: timeout_ms must be positive");
  cudaStream_t s = (cudaStream_t)stream;
  cudaEvent_t mark = mg->mark;
  cudaError_t err = cudaEventRecord(mark, s);
  if (err != cudaSuccess) return cuda_fail(mg->ctx, err, "mgpu: record sync mark");
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    err = cudaEventQuery(mark);
    if (err == cudaSuccess) break;
    if (err != cudaErrorNotReady) return cuda_fail(mg->ctx, err, "mgpu: sync");
    ncclResult_t r = ncclSuccess;
    nccl().async_error(mg->comm, &r);
    if (r != ncclSuccess && r != ncclInProgress) {
      nccl().abort(mg->comm);
      mg->broken = true;
      return nccl_fail(mg, r, "mgpu: collective failed");
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      nccl().abort(mg->comm);
      mg->broken = true;
      return fail(mg->ctx, B2K_ETIMEOUT, "mgpu: step not finished within %lld ms (communicator aborted)",
                  (long long)timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  return b2k_stream_sync(mg->ctx, stream);
}

int b2k_mgpu_gemm_tf32x3(b2k_mgpu *mg, const float *a_rows, const float *b, float *c, int64_t m, int64_t n,
                         int64_t k, int64_t align, int32_t b_layout, const float *bias, int32_t relu, int32_t panels,
                         void *stream) {
  int rc = check_handle(mg);
  if (rc) return rc;
  b2k_ctx *ctx = mg->ctx;
  if (m <= 0 || n <= 0 || k <= 0 || align <= 0 || !c || (b_layout != B2K_B_KN && b_layout != B2K_B_NK))
    return fail(ctx, B2K_EINVAL, "mgpu gemm: bad shape or layout");
  if (panels < 1 || panels > kMaxSplits || panels > n)
    return fail(ctx, B2K_EINVAL, "mgpu gemm: panels must be in 1..min(%d, n)", kMaxSplits);
  if (mg->rank == 0 && !b) return fail(ctx, B2K_EINVAL, "mgpu gemm: B is required on rank 0");
  cudaStream_t s = (cudaStream_t)stream;
  const int world = mg->world;
  const Part mine = part_of(m, world, mg->rank, align);
  if (mine.count > 0 && !a_rows) return fail(ctx, B2K_EINVAL, "mgpu gemm: A rows missing");
  int64_t width = 0;
  bool equal = true;
  for (int r = 0; r < world; ++r) {
    const Part p = part_of(m, world, r, align);
    width = std::max(width, p.count);
    equal = equal && p.count == part_of(m, world, 0, align).count;
  }
  // staging: B panels (k * n), this rank's C panels (width * n), gathered
  // panels (world * width * n); one panel with equal shards needs only B
  const bool direct = panels == 1 && equal;
  rc = reserve(mg, (size_t)(k * n + (direct ? 0 : (world + 1) * width * n)), s);
  if (rc) return rc;
  float *bstage = mg->ws;
  float *cstage = bstage + k * n;
  float *gathered = cstage + width * n;
  rc = begin(mg, s);
  if (rc) return rc;
  std::vector<Part> cols(panels);
  for (int p = 0; p < panels; ++p) cols[p] = part_of(n, panels, p, 1);
  // Broadcast every panel at once: they run in order on the communicator's
  // stream; panel p's GEMM waits only for panel p.  A [K, N] B is packed
  // panel by panel on rank 0 (its columns are strided); an [N, K] B's panels
  // are contiguous rows.  One panel is the whole contiguous B: rank 0
  // broadcasts it in place from the caller's buffer (NCCL's root only reads
  // an in-place buffer) and multiplies from there, with no staging copy
  // ahead of the broadcast.
  const bool b_in_place = panels == 1 && mg->rank == 0;
  const float *bsrc = b_in_place ? b : bstage;
  for (int p = 0; p < panels; ++p) {
    const int64_t w = cols[p].count;
    float *dst = b_in_place ? const_cast<float *>(b) : bstage + cols[p].start * k;  // panel p: [k][w] or [w][k]
    if (mg->rank == 0 && !b_in_place) {
      cudaError_t err = b_layout == B2K_B_KN
                            ? cudaMemcpy2DAsync(dst, w * sizeof(float), b + cols[p].start, n * sizeof(float),
                                                w * sizeof(float), k, cudaMemcpyDeviceToDevice, mg->comm_stream)
                            : cudaMemcpyAsync(dst, b + cols[p].start * k, (size_t)(w * k) * sizeof(float),
                                              cudaMemcpyDeviceToDevice, mg->comm_stream);
      rc = cuda_ok(mg, err, "mgpu gemm: stage B panel");
      if (rc) return rc;
    }
    if (world > 1) {
      rc = settle(mg, nccl().broadcast(dst, dst, (size_t)(w * k), ncclFloat32, 0, mg->comm, mg->comm_stream),
                  "ncclBroadcast");
      if (rc) return rc;
    }
    rc = cuda_ok(mg, cudaEventRecord(mg->ready[p], mg->comm_stream), "mgpu gemm: record panel");
    if (rc) return rc;
  }
  for (int p = 0; p < panels; ++p) {
    const int64_t w = cols[p].count;
    rc = cuda_ok(mg, cudaStreamWaitEvent(s, mg->ready[p], 0), "mgpu gemm: wait panel");
    if (rc) return rc;
    if (mine.count > 0) {
      float *dst = direct ? c + mine.start * n : cstage + cols[p].start * width;
      rc = b2k_gemm_tf32x3(ctx, a_rows, bsrc + cols[p].start * k, dst, mine.count, w, k, k,
                           b_layout == B2K_B_KN ? w : k, direct ? n : w, b_layout,
                           bias ? bias + cols[p].start : nullptr, relu, s);
      if (rc) return rc;
    }
    rc = cuda_ok(mg, cudaEventRecord(mg->computed[p], s), "mgpu gemm: record GEMM");
    if (rc) return rc;
  }
  if (direct) {
    rc = gather_rows(mg, c, m, align, n, 1, nullptr);
    if (rc) return rc;
    return finish(mg, s);
  }
  // panel p of every rank: [width][w] (padded rows for uneven shards) ->
  // gathered [world][width][w] -> C[rows of rank r][columns of p]
  for (int p = 0; p < panels; ++p) {
    const int64_t w = cols[p].count;
    rc = cuda_ok(mg, cudaStreamWaitEvent(mg->comm_stream, mg->computed[p], 0), "mgpu gemm: wait GEMM");
    if (rc) return rc;
    float *send = cstage + cols[p].start * width;
    float *recv = gathered + cols[p].start * width * world;
    if (world > 1) {
      rc = settle(mg, nccl().all_gather(send, recv, (size_t)(width * w), ncclFloat32, mg->comm, mg->comm_stream),
                  "ncclAllGather");
      if (rc) return rc;
    }
    for (int r = 0; r < world; ++r) {
      const Part pr = part_of(m, world, r, align);
      if (pr.count == 0) continue;
      const float *src = world > 1 ? recv + (size_t)r * width * w : send;
      rc = cuda_ok(mg, cudaMemcpy2DAsync(c + pr.start * n + cols[p].start, n * sizeof(float), src, w * sizeof(float),
                                         w * sizeof(float), pr.count, cudaMemcpyDeviceToDevice, mg->comm_stream),
                   "mgpu gemm: place C panel");
      if (rc) return rc;
    }
  }
  return finish(mg, s);
}

int b2k_mgpu_row_softmax_f32(b2k_mgpu *mg, const float *x_rows, float *y, int64_t rows, int64_t cols,
                             int32_t pieces, void *stream) {
  int rc = check_handle(mg);
  if (rc) return rc;
  if (rows <= 0 || cols <= 0 || !y) return fail(mg->ctx, B2K_EINVAL, "mgpu softmax: bad shape");
  const Part mine = part_of(rows, mg->world, mg->rank, 1);
  if (mine.count > 0 && !x_rows) return fail(mg->ctx, B2K_EINVAL, "mgpu softmax: x rows missing");
  cudaStream_t s = (cudaStream_t)stream;
  return run_slabs(mg, y, rows, 1, cols, pieces, s, [&](int64_t at, int64_t count) {
    return b2k_row_softmax_f32(mg->ctx, x_rows + at * cols, y + (mine.start + at) * cols, count, cols, cols, cols,
                               s);
  });
}

int b2k_mgpu_pointwise_f32(b2k_mgpu *mg, const b2k_pw_program *program, const float *const *inputs, float *out,
                           int64_t n, int64_t align, int32_t pieces, void *stream) {
  int rc = check_handle(mg);
  if (rc) return rc;
  if (!program || !inputs || !out || n <= 0 || align <= 0 || program->n_inputs < 0 ||
      program->n_inputs > B2K_PW_MAX_INPUTS)
    return fail(mg->ctx, B2K_EINVAL, "mgpu pointwise: bad arguments");
  const Part mine = part_of(n, mg->world, mg->rank, align);
  cudaStream_t s = (cudaStream_t)stream;
  return run_slabs(mg, out, n, align, 1, pieces, s, [&](int64_t at, int64_t count) {
    const float *moved[B2K_PW_MAX_INPUTS];
    for (int r = 0; r < program->n_inputs; ++r) moved[r] = program->broadcast[r] ? inputs[r] : inputs[r] + at;
    return b2k_pointwise_f32(mg->ctx, program, moved, out + mine.start + at, count, s);
  });
}

int b2k_mgpu_attention_tf32x3(b2k_mgpu *mg, const float *q, const float *k, const float *v, float *o, int64_t bh,
                              int64_t s_q, int64_t s_kv, int64_t d, int64_t dv, float scale_div, int32_t pieces,
                              void *stream) {
  int rc = check_handle(mg);
  if (rc) return rc;
  if (bh <= 0 || s_q <= 0 || s_kv <= 0 || d <= 0 || dv <= 0 || !o)
    return fail(mg->ctx, B2K_EINVAL, "mgpu attention: bad shape");
  const Part mine = part_of(bh, mg->world, mg->rank, 1);
  if (mine.count > 0 && (!q || !k || !v)) return fail(mg->ctx, B2K_EINVAL, "mgpu attention: Q, K, V heads missing");
  cudaStream_t s = (cudaStream_t)stream;
  return run_slabs(mg, o, bh, 1, s_q * dv, pieces, s, [&](int64_t at, int64_t count) {
    return b2k_attention_tf32x3(mg->ctx, q + at * s_q * d, k + at * s_kv * d, v + at * s_kv * dv,
                                o + (mine.start + at) * s_q * dv, count, s_q, s_kv, d, dv, scale_div, nullptr,
                                B2K_K_SD, s);
  });
}

}  // extern "C"
