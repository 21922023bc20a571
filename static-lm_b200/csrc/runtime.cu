// runtime.cu -- the C ABI of include/slm_b200.h: device arena, uploaded Q4_0
// weights, the operator entry points and the model driver (prefill, batched
// decode, greedy generation, embeddings) with CUDA-graph replay of decode.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types and prototypes only: the library is resolved at run time

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <utility>
#include <vector>

#include "../../include/slm_b200.h"
#include "async.cuh"
#include "kernels.h"

using namespace slm;

// The library is built with -fvisibility=hidden; only the C ABI is exported.
#define SLM_EXPORT extern "C" __attribute__((visibility("default")))

// ============================================================== errors

namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}

#define CUDA_TRY(call)                                                                  \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return fail(SLM_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

#define TRY(expr)                   \
    do {                            \
        int rc_ = (expr);           \
        if (rc_ != SLM_OK) return rc_; \
    } while (0)

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

constexpr uint64_t ARENA_ALIGN_F32 = 16;  // 64 bytes (arena.rs:6-7)

inline uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

int launch_check(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SLM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return SLM_OK;
}

// kernels with more than 48 KB of dynamic shared memory need an opt-in once
// per device
void ensure_kernel_attributes();

}  // namespace

// ============================================================== arena

struct slm_arena {
    int device;
    float *base;
    uint64_t capacity;
    uint64_t cursor;
};

namespace {

bool slice_ok(const slm_arena *a, slm_slice s) {
    return s.offset <= a->capacity && s.len <= a->capacity - s.offset;
}

bool overlaps(slm_slice a, slm_slice b) {
    return a.offset < b.offset + b.len && b.offset < a.offset + a.len;
}

}  // namespace

SLM_EXPORT const char *slm_last_error(void) { return g_err.c_str(); }
SLM_EXPORT const char *slm_version(void) { return "static-lm-b200 0.1 (sm_100a)"; }

SLM_EXPORT int slm_arena_create(int device, uint64_t capacity, slm_arena **out) {
    if (!out) return fail(SLM_ERR_INVALID_ARG, "slm_arena_create: out is null");
    *out = nullptr;
    DeviceScope ds(device);
    uint64_t cap = round_up(std::max<uint64_t>(capacity, ARENA_ALIGN_F32), ARENA_ALIGN_F32);
    float *p = nullptr;
    CUDA_TRY(cudaMalloc(&p, cap * sizeof(float)));
    cudaError_t e = cudaMemset(p, 0, cap * sizeof(float));
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(SLM_ERR_CUDA, std::string("cudaMemset: ") + cudaGetErrorString(e));
    }
    *out = new slm_arena{device, p, cap, 0};
    return SLM_OK;
}

SLM_EXPORT void slm_arena_destroy(slm_arena *a) {
    if (!a) return;
    DeviceScope ds(a->device);
    cudaFree(a->base);
    delete a;
}

SLM_EXPORT int slm_arena_alloc_slice(slm_arena *a, uint64_t len, slm_slice *out) {
    if (!a || !out) return fail(SLM_ERR_INVALID_ARG, "slm_arena_alloc_slice: null argument");
    uint64_t off = round_up(a->cursor, ARENA_ALIGN_F32);
    if (off > a->capacity || len > a->capacity - off)
        return fail(SLM_ERR_CAPACITY, "AlignedArena out of capacity: requested " +
                                          std::to_string(len) + " elements at offset " +
                                          std::to_string(off) + ", capacity " +
                                          std::to_string(a->capacity));
    a->cursor = off + len;
    *out = slm_slice{off, len};
    return SLM_OK;
}

SLM_EXPORT int slm_arena_alloc_q8_scratch(slm_arena *a, uint64_t num_blocks, slm_slice *out) {
    return slm_arena_alloc_slice(a, (q8x_bytes(num_blocks) + 3) / 4, out);
}

SLM_EXPORT void slm_arena_reset(slm_arena *a) {
    if (a) a->cursor = 0;
}
SLM_EXPORT uint64_t slm_arena_capacity(const slm_arena *a) { return a ? a->capacity : 0; }
SLM_EXPORT uint64_t slm_arena_used(const slm_arena *a) { return a ? a->cursor : 0; }

SLM_EXPORT float *slm_arena_device_ptr(slm_arena *a, slm_slice s) {
    if (!a || !slice_ok(a, s)) {
        fail(SLM_ERR_OUT_OF_BOUNDS, "ArenaSlice out of bounds");
        return nullptr;
    }
    return a->base + s.offset;
}

SLM_EXPORT int slm_arena_write(slm_arena *a, slm_slice s, const float *host, uint64_t n) {
    if (!a || (!host && n)) return fail(SLM_ERR_INVALID_ARG, "slm_arena_write: null argument");
    if (!slice_ok(a, s)) return fail(SLM_ERR_OUT_OF_BOUNDS, "ArenaSlice out of bounds");
    if (n != s.len) return fail(SLM_ERR_SHAPE, "slm_arena_write: length mismatch");
    DeviceScope ds(a->device);
    CUDA_TRY(cudaMemcpy(a->base + s.offset, host, n * sizeof(float), cudaMemcpyHostToDevice));
    return SLM_OK;
}

SLM_EXPORT int slm_arena_read(slm_arena *a, slm_slice s, float *host, uint64_t n) {
    if (!a || (!host && n)) return fail(SLM_ERR_INVALID_ARG, "slm_arena_read: null argument");
    if (!slice_ok(a, s)) return fail(SLM_ERR_OUT_OF_BOUNDS, "ArenaSlice out of bounds");
    if (n != s.len) return fail(SLM_ERR_SHAPE, "slm_arena_read: length mismatch");
    DeviceScope ds(a->device);
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(host, a->base + s.offset, n * sizeof(float), cudaMemcpyDeviceToHost));
    return SLM_OK;
}

// ============================================================== Q4_0 weights

namespace {

// 576-byte row tiles -> BlockQ4_0 rows [rows x cols/32] (18 B each), the
// inverse of the device repack (repack_q4_kernel).
void unpack_rows(const uint8_t *tiles, uint64_t rows, uint64_t nb, uint8_t *dst) {
    for (uint64_t r = 0; r < rows; r++) {
        uint64_t t = r / TILE_ROWS, lane = r % TILE_ROWS;
        for (uint64_t j = 0; j < nb; j++) {
            uint8_t *blk = dst + (r * nb + j) * 18;
            const uint8_t *tp = tiles + tile_offset(t, nb, j);
            std::memcpy(blk, tp + 512 + lane * 2, 2);
            std::memcpy(blk + 2, tp + lane * 16, 16);
        }
    }
}

uint64_t tiled_bytes(uint64_t rows, uint64_t cols) {
    return (rows + TILE_ROWS - 1) / TILE_ROWS * (cols / QK) * TILE_BYTES;
}

// Host -> device path of Q4_0 weights: the caller's blocks (typically the
// mmap'd GGUF tensor, GgufFile::tensor_q4_0, loader.rs:496-500) are copied in
// chunks into one of two pinned staging buffers, sent with cudaMemcpyAsync
// into a device scratch of the same size, and repacked into the row tiles by
// a kernel; while the GPU copies and repacks one chunk, the host fills the
// other staging buffer.  Host memory is never repacked or held whole.
class Q4Uploader {
  public:
    static constexpr size_t CHUNK = 8u << 20;  // bytes per staging buffer
    ~Q4Uploader() { release(); }
    int begin() {
        CUDA_TRY(cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking));
        for (int i = 0; i < 2; i++) {
            CUDA_TRY(cudaMallocHost(&host_[i], CHUNK));
            CUDA_TRY(cudaMalloc(&dev_[i], CHUNK));
            CUDA_TRY(cudaEventCreateWithFlags(&done_[i], cudaEventDisableTiming));
        }
        return SLM_OK;
    }
    // rows [row0, row0+nrows) of a tiled matrix of nb blocks per row from
    // nrows*nb host blocks
    int rows(const void *src, uint64_t nrows, uint64_t nb, uint64_t row0, uint8_t *tiles) {
        const uint64_t row_bytes = nb * 18;
        const uint64_t per_chunk = std::max<uint64_t>(1, CHUNK / row_bytes);
        if (per_chunk * row_bytes > CHUNK) return fail(SLM_ERR_SHAPE, "a Q4_0 row exceeds the staging buffer");
        for (uint64_t r = 0; r < nrows; r += per_chunk) {
            const uint64_t n = std::min(per_chunk, nrows - r);
            const int b = next_++ & 1;
            CUDA_TRY(cudaEventSynchronize(done_[b]));  // the buffer's previous chunk has been sent
            std::memcpy(host_[b], static_cast<const uint8_t *>(src) + r * row_bytes, n * row_bytes);
            CUDA_TRY(cudaMemcpyAsync(dev_[b], host_[b], n * row_bytes, cudaMemcpyHostToDevice, st_));
            launch_repack_q4(dev_[b], n, (int)nb, row0 + r, tiles, st_);
            CUDA_TRY(cudaGetLastError());
            CUDA_TRY(cudaEventRecord(done_[b], st_));
        }
        return SLM_OK;
    }
    cudaStream_t stream() const { return st_; }
    int finish() {
        CUDA_TRY(cudaStreamSynchronize(st_));
        return SLM_OK;
    }
    void release() {
        if (st_) cudaStreamSynchronize(st_);
        for (int i = 0; i < 2; i++) {
            if (host_[i]) cudaFreeHost(host_[i]);
            if (dev_[i]) cudaFree(dev_[i]);
            if (done_[i]) cudaEventDestroy(done_[i]);
            host_[i] = nullptr;
            dev_[i] = nullptr;
            done_[i] = nullptr;
        }
        if (st_) cudaStreamDestroy(st_);
        st_ = nullptr;
    }

  private:
    cudaStream_t st_ = nullptr;
    void *host_[2] = {nullptr, nullptr};
    void *dev_[2] = {nullptr, nullptr};
    cudaEvent_t done_[2] = {nullptr, nullptr};
    unsigned next_ = 0;
};

}  // namespace

struct slm_qmatrix {
    int device;
    uint8_t *tiles;
    uint64_t rows, cols, bytes;
};

SLM_EXPORT int slm_qmatrix_upload(int device, const void *blocks, uint64_t rows, uint64_t cols,
                                  slm_qmatrix **out) {
    if (!blocks || !out) return fail(SLM_ERR_INVALID_ARG, "slm_qmatrix_upload: null argument");
    *out = nullptr;
    if (cols == 0 || cols % QK) return fail(SLM_ERR_SHAPE, "cols must be a multiple of 32");
    if (rows == 0) return fail(SLM_ERR_SHAPE, "rows must be positive");
    if ((uintptr_t)blocks & 1) return fail(SLM_ERR_INVALID_ARG, "Q4_0 blocks must be 2-byte aligned");
    DeviceScope ds(device);
    uint64_t bytes = tiled_bytes(rows, cols);
    uint8_t *d = nullptr;
    CUDA_TRY(cudaMalloc(&d, bytes));
    Q4Uploader up;
    int rc = up.begin();
    if (rc == SLM_OK && cudaMemsetAsync(d, 0, bytes, up.stream()) != cudaSuccess)  // rows past the last
        rc = fail(SLM_ERR_CUDA, "cudaMemsetAsync");
    if (rc == SLM_OK) rc = up.rows(blocks, rows, cols / QK, 0, d);
    if (rc == SLM_OK) rc = up.finish();
    if (rc != SLM_OK) {
        up.release();
        cudaFree(d);
        return rc;
    }
    *out = new slm_qmatrix{device, d, rows, cols, bytes};
    return SLM_OK;
}

SLM_EXPORT int slm_qmatrix_download(const slm_qmatrix *w, void *blocks_out) {
    if (!w || !blocks_out) return fail(SLM_ERR_INVALID_ARG, "slm_qmatrix_download: null argument");
    DeviceScope ds(w->device);
    std::vector<uint8_t> host(w->bytes);
    CUDA_TRY(cudaMemcpy(host.data(), w->tiles, w->bytes, cudaMemcpyDeviceToHost));
    unpack_rows(host.data(), w->rows, w->cols / QK, (uint8_t *)blocks_out);
    return SLM_OK;
}

SLM_EXPORT void slm_qmatrix_destroy(slm_qmatrix *w) {
    if (!w) return;
    DeviceScope ds(w->device);
    cudaFree(w->tiles);
    delete w;
}

// ============================================================== operators

namespace {

int gemm_into(const slm_qmatrix *w, Q8X x, float *out, uint64_t batch, uint64_t rows,
              uint64_t cols, cudaStream_t st, bool tc = false) {
    ensure_kernel_attributes();
    GemvArgs g{};
    g.tc = tc;
    g.w = w->tiles;
    g.rows = (int)rows;
    g.nb = (int)(cols / QK);
    g.x = x;
    g.batch = (int)batch;
    g.epi = EPI_STORE;
    g.out = out;
    g.ld_out = rows;
    launch_gemv(g, st);
    return launch_check("gemv kernel");
}

int check_gemm_shape(const slm_qmatrix *w, uint64_t batch, uint64_t rows, uint64_t cols) {
    if (!w) return fail(SLM_ERR_INVALID_ARG, "weights are null");
    if (cols % QK) return fail(SLM_ERR_SHAPE, "cols must be a multiple of 32");
    if (w->rows != rows || w->cols != cols)
        return fail(SLM_ERR_SHAPE, "weights block count mismatch");
    if (batch > (uint64_t)INT32_MAX || rows > (uint64_t)INT32_MAX)
        return fail(SLM_ERR_SHAPE, "batch/rows too large");
    return SLM_OK;
}

}  // namespace

SLM_EXPORT int slm_gemm_q4_0_arena(slm_arena *a, const slm_qmatrix *w, slm_slice in,
                                   slm_slice q8, slm_slice outs, uint64_t batch, uint64_t rows,
                                   uint64_t cols, void *stream) {
    if (!a) return fail(SLM_ERR_INVALID_ARG, "arena is null");
    TRY(check_gemm_shape(w, batch, rows, cols));
    if (in.len != batch * cols) return fail(SLM_ERR_SHAPE, "inputs batch size mismatch");
    if (outs.len != batch * rows) return fail(SLM_ERR_SHAPE, "output batch size mismatch");
    if (!slice_ok(a, in) || !slice_ok(a, q8) || !slice_ok(a, outs))
        return fail(SLM_ERR_OUT_OF_BOUNDS, "ArenaSlice out of bounds");
    if (overlaps(in, q8) || overlaps(in, outs) || overlaps(q8, outs))
        return fail(SLM_ERR_OVERLAP, "gemv_slices: slices must be pairwise disjoint");
    uint64_t blocks = batch * (cols / QK);
    if (q8x_bytes(blocks) > q8.len * 4) return fail(SLM_ERR_CAPACITY, "q8_scratch slice too small");
    if (w->device != a->device) return fail(SLM_ERR_INVALID_ARG, "weights on another device");
    if (batch == 0 || rows == 0) return SLM_OK;
    DeviceScope ds(a->device);
    cudaStream_t st = (cudaStream_t)stream;
    Q8X x = q8x_view(a->base + q8.offset, blocks);
    launch_quantize_q8x(a->base + in.offset, cols, (int)cols, x, (int)batch, st);
    TRY(launch_check("quantize kernel"));
    return gemm_into(w, x, a->base + outs.offset, batch, rows, cols, st);
}

SLM_EXPORT int slm_gemv_q4_0_arena(slm_arena *a, const slm_qmatrix *w, slm_slice in, slm_slice q8,
                                   slm_slice out, uint64_t rows, uint64_t cols, void *stream) {
    if (out.len != rows) return fail(SLM_ERR_SHAPE, "output length mismatch");
    if (in.len != cols) return fail(SLM_ERR_SHAPE, "input length mismatch");
    return slm_gemm_q4_0_arena(a, w, in, q8, out, 1, rows, cols, stream);
}

SLM_EXPORT uint64_t slm_gemm_q4_0_scratch_bytes(uint64_t batch, uint64_t cols) {
    return q8x_bytes(batch * (cols / QK));
}

SLM_EXPORT int slm_gemm_q4_0(const slm_qmatrix *w, const void *xq, float *out, uint64_t batch,
                             uint64_t rows, uint64_t cols, void *scratch, uint64_t scratch_bytes,
                             void *stream) {
    TRY(check_gemm_shape(w, batch, rows, cols));
    if (batch == 0 || rows == 0) return SLM_OK;
    if (!xq || !out || !scratch) return fail(SLM_ERR_INVALID_ARG, "null device pointer");
    uint64_t blocks = batch * (cols / QK);
    if (scratch_bytes < q8x_bytes(blocks)) return fail(SLM_ERR_CAPACITY, "scratch too small");
    if ((uintptr_t)scratch % 16) return fail(SLM_ERR_INVALID_ARG, "scratch must be 16-byte aligned");
    DeviceScope ds(w->device);
    cudaStream_t st = (cudaStream_t)stream;
    Q8X x = q8x_view(scratch, blocks);
    launch_q8_ref_to_q8x(xq, x, blocks, st);
    TRY(launch_check("q8 conversion kernel"));
    return gemm_into(w, x, out, batch, rows, cols, st);
}

SLM_EXPORT int slm_gemm_q4_0_tensor_cores(const slm_qmatrix *w, const void *xq, float *out, uint64_t batch,
                                          uint64_t rows, uint64_t cols, void *scratch, uint64_t scratch_bytes,
                                          void *stream) {
    TRY(check_gemm_shape(w, batch, rows, cols));
    if (batch == 0 || rows == 0) return SLM_OK;
    if (!xq || !out || !scratch) return fail(SLM_ERR_INVALID_ARG, "null device pointer");
    uint64_t blocks = batch * (cols / QK);
    if (scratch_bytes < q8x_bytes(blocks)) return fail(SLM_ERR_CAPACITY, "scratch too small");
    if ((uintptr_t)scratch % 16) return fail(SLM_ERR_INVALID_ARG, "scratch must be 16-byte aligned");
    DeviceScope ds(w->device);
    cudaStream_t st = (cudaStream_t)stream;
    Q8X x = q8x_view(scratch, blocks);
    launch_q8_ref_to_q8x(xq, x, blocks, st);
    TRY(launch_check("q8 conversion kernel"));
    return gemm_into(w, x, out, batch, rows, cols, st, true);
}

// ---- the allocation-free GEMM: Q8 activations in a static device buffer

namespace {

// Lives in this library's device image on every device that loads it; the
// quantize kernel writes every block the GEMV then reads, so nothing in it
// has to start at zero and stale contents from an earlier call are never read.
static __device__ __align__(256) unsigned char g_noalloc_q8[SLM_NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[NOALLOC_MAX_DEVICES];  // device address per device, null until looked up

// The buffer's address on the current device (looked up once per device,
// with that device current).
int noalloc_scratch(int device, void **out) {
    if (device < 0 || device >= NOALLOC_MAX_DEVICES)
        return fail(SLM_ERR_INVALID_ARG, "device ordinal out of range for the static scratch");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_q8);
        if (e != cudaSuccess)
            return fail(SLM_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_noalloc_ptr[device] = p;
    }
    *out = g_noalloc_ptr[device];
    return SLM_OK;
}

}  // namespace

SLM_EXPORT int slm_gemm_q4_0_f32_noalloc(const slm_qmatrix *w, const float *inputs_dev,
                                         float *output_dev, uint64_t batch, uint64_t rows,
                                         uint64_t cols, void *stream) {
    TRY(check_gemm_shape(w, batch, rows, cols));
    if (batch == 0 || rows == 0) return SLM_OK;
    if (!inputs_dev || !output_dev) return fail(SLM_ERR_INVALID_ARG, "null device pointer");
    const uint64_t blocks = batch * (cols / QK);
    if (q8x_bytes(blocks) > SLM_NOALLOC_SCRATCH_BYTES)
        return fail(SLM_ERR_CAPACITY,
                    "batch*cols needs " + std::to_string(q8x_bytes(blocks)) +
                        " bytes of Q8 scratch; the static buffer holds " +
                        std::to_string(SLM_NOALLOC_SCRATCH_BYTES));
    DeviceScope ds(w->device);
    void *scratch = nullptr;
    TRY(noalloc_scratch(w->device, &scratch));
    cudaStream_t st = (cudaStream_t)stream;
    Q8X x = q8x_view(scratch, blocks);
    launch_quantize_q8x(inputs_dev, cols, (int)cols, x, (int)batch, st);
    TRY(launch_check("quantize kernel"));
    return gemm_into(w, x, output_dev, batch, rows, cols, st);
}

SLM_EXPORT int slm_selftest_bounded_wait(int device, uint64_t limit_cycles) {
    if (limit_cycles == 0 || limit_cycles > (uint64_t)WAIT_LIMIT)
        return fail(SLM_ERR_INVALID_ARG, "limit_cycles must be in [1, 2e9]");
    DeviceScope ds(device);
    int32_t *err = nullptr, host = 0;
    CUDA_TRY(cudaMalloc(&err, sizeof(int32_t)));
    cudaError_t e = cudaMemset(err, 0, sizeof(int32_t));
    if (e == cudaSuccess) {
        launch_wait_selftest((long long)limit_cycles, err, 0);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(&host, err, sizeof(int32_t), cudaMemcpyDeviceToHost);
    cudaFree(err);
    if (e != cudaSuccess) return fail(SLM_ERR_CUDA, std::string("wait self-test: ") + cudaGetErrorString(e));
    if (host == 3) return fail(SLM_ERR_DEVICE_INPUT, "a device wait timed out");
    return fail(SLM_ERR_CUDA, "wait self-test: the wait did not report its timeout");
}

SLM_EXPORT int slm_quantize_row_q8_0(const float *src, void *dst, uint64_t n, void *stream) {
    if (n % QK) return fail(SLM_ERR_SHAPE, "src length must be a multiple of 32");
    if (n == 0) return SLM_OK;
    if (!src || !dst) return fail(SLM_ERR_INVALID_ARG, "null device pointer");
    launch_quantize_q8_ref(src, dst, n, (cudaStream_t)stream);
    return launch_check("quantize kernel");
}

SLM_EXPORT int slm_exec_rmsnorm(const float *const *in, float *out, uint64_t len, float eps,
                                void *stream) {
    if (!in || !in[0] || !in[1] || !out) return fail(SLM_ERR_INVALID_ARG, "null pointer");
    launch_rmsnorm_vec(in[0], in[1], out, len, eps, (cudaStream_t)stream);
    return launch_check("rmsnorm kernel");
}

SLM_EXPORT int slm_exec_softmax(const float *const *in, float *out, uint64_t len, void *stream) {
    if (!in || !in[0] || !out) return fail(SLM_ERR_INVALID_ARG, "null pointer");
    launch_softmax_vec(in[0], out, len, (cudaStream_t)stream);
    return launch_check("softmax kernel");
}

SLM_EXPORT int slm_exec_swiglu(const float *const *in, float *out, uint64_t len, void *stream) {
    if (!in || !in[0] || !in[1] || !out) return fail(SLM_ERR_INVALID_ARG, "null pointer");
    launch_swiglu_vec(in[0], in[1], out, len, (cudaStream_t)stream);
    return launch_check("swiglu kernel");
}

SLM_EXPORT int slm_exec_residual_add(const float *const *in, float *out, uint64_t len,
                                     void *stream) {
    if (!in || !in[0] || !in[1] || !out) return fail(SLM_ERR_INVALID_ARG, "null pointer");
    launch_residual_add_vec(in[0], in[1], out, len, (cudaStream_t)stream);
    return launch_check("residual kernel");
}

SLM_EXPORT int slm_exec_l2_norm(const float *const *in, float *out, uint64_t len, float eps,
                                void *stream) {
    if (!in || !in[0] || !out) return fail(SLM_ERR_INVALID_ARG, "null pointer");
    launch_l2norm_vec(in[0], out, len, eps, (cudaStream_t)stream);
    return launch_check("l2norm kernel");
}

// ---- JitKernelFn-compatible entry points (engine.rs:15, 66-72)

namespace {

// One compiled graph: the operator, the constants FuseGraph bakes in (n, eps)
// and the stream the returned function enqueues on.
struct JitSlot {
    int op = -1;
    uint64_t n = 0;
    float eps = 0.0f;
    float inv_n = 0.0f;
    cudaStream_t stream = nullptr;
};
constexpr int JIT_SLOTS = 64;
JitSlot g_jit[JIT_SLOTS];
std::mutex g_jit_mu;

void jit_run(int i, const float *const *in, float *out, size_t len) {
    const JitSlot &k = g_jit[i];
    if (!in || !out || len == 0) return;
    switch (k.op) {
        case SLM_JIT_RMSNORM: launch_rmsnorm_vec_inv_n(in[0], in[1], out, len, k.eps, k.inv_n, k.stream); break;
        case SLM_JIT_SOFTMAX: launch_softmax_vec(in[0], out, len, k.stream); break;
        case SLM_JIT_SWIGLU: launch_swiglu_vec(in[0], in[1], out, len, k.stream); break;
        case SLM_JIT_RESIDUAL_ADD: launch_residual_add_vec(in[0], in[1], out, len, k.stream); break;
        case SLM_JIT_L2_NORM: launch_l2norm_vec(in[0], out, len, k.eps, k.stream); break;
        default: break;
    }
    launch_check("JIT kernel");  // a launch failure is left in slm_last_error()
}

// a distinct plain C function per slot, so that each carries its constants
// without a closure argument
template <int I>
void jit_entry(const float *const *in, float *out, size_t len) {
    jit_run(I, in, out, len);
}
template <int... I>
constexpr std::array<slm_jit_kernel_fn, sizeof...(I)> jit_table(std::integer_sequence<int, I...>) {
    return {&jit_entry<I>...};
}
const std::array<slm_jit_kernel_fn, JIT_SLOTS> g_jit_fn = jit_table(std::make_integer_sequence<int, JIT_SLOTS>{});

}  // namespace

SLM_EXPORT int slm_jit_compile(int op, uint64_t n, float eps, void *stream, slm_jit_kernel_fn *kernel_out) {
    if (!kernel_out) return fail(SLM_ERR_INVALID_ARG, "kernel_out is null");
    if (op < SLM_JIT_RMSNORM || op > SLM_JIT_L2_NORM) return fail(SLM_ERR_INVALID_ARG, "unknown JIT operator");
    if (op == SLM_JIT_RMSNORM && n == 0) return fail(SLM_ERR_INVALID_ARG, "rmsnorm needs n > 0");
    // constants the operator does not use do not tell graphs apart
    if (op != SLM_JIT_RMSNORM) n = 0;
    if (op != SLM_JIT_RMSNORM && op != SLM_JIT_L2_NORM) eps = 0.0f;
    std::lock_guard<std::mutex> lock(g_jit_mu);
    int free_slot = -1;
    for (int i = 0; i < JIT_SLOTS; i++) {
        const JitSlot &k = g_jit[i];
        if (k.op < 0) {
            if (free_slot < 0) free_slot = i;
            continue;
        }
        // the engine's cache: the same graph gives the same function
        if (k.op == op && k.n == n && std::memcmp(&k.eps, &eps, sizeof(float)) == 0 &&
            k.stream == (cudaStream_t)stream) {
            *kernel_out = g_jit_fn[i];
            return SLM_OK;
        }
    }
    if (free_slot < 0) return fail(SLM_ERR_CAPACITY, "all 64 JIT kernel slots are in use");
    JitSlot &k = g_jit[free_slot];
    k.op = op;
    k.n = n;
    k.eps = eps;
    k.inv_n = n ? 1.0f / (float)n : 0.0f;  // FuseGraph::rmsnorm: 1.0 / (n as f32)
    k.stream = (cudaStream_t)stream;
    *kernel_out = g_jit_fn[free_slot];
    return SLM_OK;
}

SLM_EXPORT int slm_rope_tables(uint32_t max_seq, uint32_t head_dim, float *cos_out,
                               float *sin_out) {
    if ((!cos_out || !sin_out) && max_seq) return fail(SLM_ERR_INVALID_ARG, "null pointer");
    if (head_dim == 0 || head_dim % 2) return fail(SLM_ERR_SHAPE, "head_dim must be even");
    uint32_t half = head_dim / 2;
    float hd_f = (float)head_dim;
    for (uint32_t pos = 0; pos < max_seq; pos++) {
        float pos_f = (float)pos;
        for (uint32_t j = 0; j < half; j++) {
            float freq = 1.0f / powf(10000.0f, (float)(2 * j) / hd_f);
            float ang = pos_f * freq;
            sin_out[(size_t)pos * half + j] = sinf(ang);
            cos_out[(size_t)pos * half + j] = cosf(ang);
        }
    }
    return SLM_OK;
}

SLM_EXPORT int slm_apply_rope_cached(float *vec, uint64_t len, const float *c, const float *s,
                                     uint32_t head_dim, void *stream) {
    if (!vec || !c || !s) return fail(SLM_ERR_INVALID_ARG, "null pointer");
    if (head_dim == 0 || head_dim % 2) return fail(SLM_ERR_SHAPE, "head_dim must be even");
    launch_rope_vec(vec, len, c, s, (int)head_dim, (cudaStream_t)stream);
    return launch_check("rope kernel");
}

namespace {

int check_config(const slm_config *c) {
    if (!c) return fail(SLM_ERR_INVALID_ARG, "config is null");
    if (c->dim == 0 || c->dim % QK) return fail(SLM_ERR_SHAPE, "dim must be a multiple of 32");
    if (c->hidden_dim == 0 || c->hidden_dim % QK)
        return fail(SLM_ERR_SHAPE, "hidden_dim must be a multiple of 32");
    if (c->num_heads == 0 || c->num_kv_heads == 0)
        return fail(SLM_ERR_SHAPE, "head counts must be positive");
    if (c->dim % c->num_heads) return fail(SLM_ERR_SHAPE, "dim must be divisible by num_heads");
    if (c->num_heads % c->num_kv_heads)
        return fail(SLM_ERR_SHAPE, "num_heads must be divisible by num_kv_heads");
    uint32_t hd = c->dim / c->num_heads;
    if (hd % 2) return fail(SLM_ERR_SHAPE, "head_dim must be even for RoPE rotation");
    if ((hd * c->num_kv_heads) % QK) return fail(SLM_ERR_SHAPE, "kv_dim must be a multiple of 32");
    if (c->num_heads / c->num_kv_heads > 32)
        return fail(SLM_ERR_SHAPE, "num_heads / num_kv_heads above 32 is not supported");
    if (c->max_seq_len == 0) return fail(SLM_ERR_SHAPE, "max_seq_len must be positive");
    if ((uint64_t)c->max_seq_len * 4 > 200 * 1024)
        return fail(SLM_ERR_SHAPE, "max_seq_len above 51200 is not supported");
    return SLM_OK;
}

// Softmax + PV form of the exact attention (AttnArgs::pv_per_head): one CTA
// per (row, query head) unless SLM_PV_PER_HEAD says otherwise (0 .. 11);
// every form gives the same results.  Unset, decode steps of at most
// CLUSTER_AUTO_ROWS rows (per part) use the one-launch cluster form (11)
// where attn_decode_cluster_preferred() says it fits (measured 30.9 against
// 34.2 us per layer at 8 rows of config 3; slower from 16 rows, and where its
// shared memory would leave the grid a second wave).
constexpr int CLUSTER_AUTO_ROWS = 8;
int env_pv_per_head() {
    const char *env = getenv("SLM_PV_PER_HEAD");
    if (!env || env[0] < '0' || env[0] > '9') return 1;
    const int v = atoi(env);
    return v <= 11 ? v : 1;
}
bool env_pv_form_auto() {
    const char *env = getenv("SLM_PV_PER_HEAD");
    return !env || env[0] < '0' || env[0] > '9';
}

AttnArgs attn_args_for(const slm_config *c) {
    AttnArgs a{};
    a.pv_per_head = env_pv_per_head();
    a.dim = (int)c->dim;
    a.num_heads = (int)c->num_heads;
    a.num_kv_heads = (int)c->num_kv_heads;
    a.head_dim = (int)(c->dim / c->num_heads);
    a.kv_dim = a.head_dim * a.num_kv_heads;
    a.max_seq = (int)c->max_seq_len;
    a.scale = 1.0f / sqrtf((float)a.head_dim);
    return a;
}

}  // namespace

SLM_EXPORT int slm_causal_attention(const float *q, const float *k, const float *v, float *att,
                                    float *out, const slm_config *cfg, uint32_t pos,
                                    void *stream) {
    TRY(check_config(cfg));
    if (!q || !k || !v || !att || !out) return fail(SLM_ERR_INVALID_ARG, "null device pointer");
    if (pos >= cfg->max_seq_len) return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence position out of bounds");
    ensure_kernel_attributes();
    AttnArgs a = attn_args_for(cfg);
    a.q = q;
    a.ldq = cfg->dim;
    a.k_base = k;
    a.v_base = v;
    a.slot = nullptr;
    a.pos = nullptr;
    a.pos_const = (int)pos;
    a.att = att;
    a.att_ld = cfg->max_seq_len;
    a.write_probs = true;
    a.out = out;
    a.ldo = cfg->dim;
    a.rows = 1;
    a.max_len = (int)pos + 1;
    // one [max_seq][kv_dim] plane of V: z = 0 for every row
    CUtensorMap vmap, kmap;
    const bool have_map = encode_v_map(&vmap, v, a.kv_dim, a.max_seq, 1, a.head_dim);
    const bool have_kmap = encode_k_map(&kmap, k, a.kv_dim, a.max_seq, 1, a.head_dim);
    launch_attention(a, have_map ? &vmap : nullptr, have_kmap ? &kmap : nullptr,
                     (cudaStream_t)stream);
    return launch_check("attention kernels");
}

SLM_EXPORT int slm_causal_attention_rows(const float *q, const float *k, const float *v, float *att,
                                         float *out, const slm_config *cfg, uint32_t n, uint32_t start_pos,
                                         int mode, void *stream) {
    TRY(check_config(cfg));
    if (!q || !k || !v || !att || !out) return fail(SLM_ERR_INVALID_ARG, "null device pointer");
    if (mode != SLM_PREFILL_EXACT && mode != SLM_PREFILL_TENSOR_CORES && mode != SLM_ATTN_FLASH_DECODE)
        return fail(SLM_ERR_INVALID_ARG, "unknown attention mode");
    if ((uint64_t)start_pos + n > cfg->max_seq_len)
        return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence position out of bounds");
    if (n == 0) return SLM_OK;
    ensure_kernel_attributes();
    cudaStream_t st = (cudaStream_t)stream;
    // row i sits at position start_pos + i (device array, as the model's rows)
    std::vector<int32_t> hpos(n);
    for (uint32_t i = 0; i < n; i++) hpos[i] = (int32_t)(start_pos + i);
    int32_t *dpos = nullptr;
    if (cudaMallocAsync((void **)&dpos, sizeof(int32_t) * n, st) != cudaSuccess)
        return fail(SLM_ERR_CUDA, "position array");
    cudaMemcpyAsync(dpos, hpos.data(), sizeof(int32_t) * n, cudaMemcpyHostToDevice, st);
    AttnArgs a = attn_args_for(cfg);
    a.q = q;
    a.ldq = cfg->dim;
    a.k_base = k;
    a.v_base = v;
    a.slot = nullptr;
    a.pos = dpos;
    a.att = att;
    a.att_ld = cfg->max_seq_len;
    a.out = out;
    a.ldo = cfg->dim;
    a.rows = (int)n;
    a.max_len = (int)(start_pos + n);
    a.prefill_run = (int)n;
    a.prefill_tc = mode == SLM_PREFILL_TENSOR_CORES;
    CUtensorMap vmap, kmap, amap;
    const bool have_v = encode_v_map(&vmap, v, a.kv_dim, a.max_seq, 1, a.head_dim);
    const bool have_k = encode_k_map(&kmap, k, a.kv_dim, a.max_seq, 1, a.head_dim);
    const bool have_a = encode_att_map(&amap, att, a.max_seq, a.num_heads, n, a.num_heads / a.num_kv_heads);
    if (mode == SLM_ATTN_FLASH_DECODE) {
        // every row as a decode row; the chunk partials in a stream-ordered
        // allocation
        a.prefill_run = 0;
        a.prefill_tc = 0;
        a.fd_nch = flash_decode_chunks(a.max_seq);
        const size_t pfloats = (size_t)n * a.num_kv_heads * a.fd_nch * (a.num_heads / a.num_kv_heads) *
                               (a.head_dim + 2);
        float *scratch = nullptr;
        if (!have_v || !have_k || cudaMallocAsync((void **)&scratch, pfloats * sizeof(float), st) != cudaSuccess) {
            cudaFreeAsync(dpos, st);
            cudaStreamSynchronize(st);
            return fail(have_v && have_k ? SLM_ERR_CUDA : SLM_ERR_SHAPE, "flash-decode set-up");
        }
        CUtensorMap kmap64;
        if (!encode_k_map(&kmap64, k, a.kv_dim, a.max_seq, 1, a.head_dim, FD_ITEM_KEYS)) {
            cudaFreeAsync(scratch, st);
            cudaFreeAsync(dpos, st);
            cudaStreamSynchronize(st);
            return fail(SLM_ERR_SHAPE, "flash-decode needs head_dim 64 or 128");
        }
        a.fd_part = scratch;
        int rc = SLM_OK;
        if (flash_decode_ok(a))
            launch_flash_decode(a, kmap64, vmap, st);
        else
            rc = fail(SLM_ERR_SHAPE, "flash-decode needs head_dim 64 or 128 and kv_mul 1, 2, 3, 4, 6 or 8");
        cudaFreeAsync(scratch, st);
        cudaFreeAsync(dpos, st);
        if (rc == SLM_OK) rc = launch_check("flash-decode attention");
        cudaStreamSynchronize(st);
        return rc;
    }
    CUtensorMap vmap_fine;
    const bool have_vf = encode_v_map(&vmap_fine, v, a.kv_dim, a.max_seq, 1, a.head_dim, V_FINE_POSITIONS);
    if (have_v && attention_fused_ok(a))
        launch_attn_fused(a, vmap, have_k ? &kmap : nullptr, have_a ? &amap : nullptr, st, nullptr,
                          have_vf ? &vmap_fine : nullptr);
    else
        launch_attention(a, have_v ? &vmap : nullptr, have_k ? &kmap : nullptr, st);
    cudaFreeAsync(dpos, st);
    const int rc = launch_check("attention kernels");
    cudaStreamSynchronize(st);  // hpos is read by the copy above
    return rc;
}

SLM_EXPORT int slm_sample_argmax(const float *logits, uint64_t n, int32_t *out, void *stream) {
    if (n == 0) return fail(SLM_ERR_INVALID_ARG, "logits cannot be empty");
    if (!logits || !out) return fail(SLM_ERR_INVALID_ARG, "null device pointer");
    if (n > (uint64_t)INT32_MAX) return fail(SLM_ERR_SHAPE, "too many logits");
    launch_argmax(logits, n, (int)n, out, 1, (cudaStream_t)stream);
    return launch_check("argmax kernel");
}

// ============================================================== model

namespace {

struct QMat {
    uint8_t *tiles = nullptr;
    int rows = 0, cols = 0;
};

struct LayerDev {
    QMat wqkv, wo, wgu, wdown;
    float *rms_att = nullptr, *rms_ffn = nullptr;
};

enum StepKind { STEP_DECODE = 0, STEP_PREFILL = 1, STEP_EMBED = 2, STEP_PREFILL_BATCH = 3 };

// NCCL entry points, looked up in whichever libnccl the process has (torch's,
// or the system's) so that the library itself has no link-time dependency.
struct NcclApi {
    decltype(&ncclGetUniqueId) get_id = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclCommGetAsyncError) async_error = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok() const {
        return get_id && init_rank_config && all_gather && destroy && abort && async_error && error_string;
    }
};

const NcclApi &nccl_api() {
    static const NcclApi api = [] {
        NcclApi a;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
        a.get_id = reinterpret_cast<decltype(a.get_id)>(dlsym(h, "ncclGetUniqueId"));
        a.init_rank_config =
            reinterpret_cast<decltype(a.init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
        a.abort = reinterpret_cast<decltype(a.abort)>(dlsym(h, "ncclCommAbort"));
        a.async_error = reinterpret_cast<decltype(a.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
        return a;
    }();
    return api;
}


}  // namespace

struct slm_model {
    int device = 0;
    cudaStream_t stream = nullptr;
    slm_config cfg{};
    int L = 0, vocab = 0, S = 0, R = 0, hd = 0, kvd = 0;
    uint8_t *wbuf = nullptr;
    uint64_t wbytes = 0;
    std::vector<LayerDev> layers;
    QMat embd, lm_head;
    float *out_norm = nullptr;
    slm_arena *arena = nullptr;
    // arena views
    float *rope_cos, *rope_sin, *x, *x_mid, *xb, *q, *logits, *att, *kv, *ybuf, *emb;
    float *tmax = nullptr;   // [R][heads][tmax_ld] per-32-key score maxima (prefill)
    int tmax_ld = 0;
    static constexpr int MAX_PARTS = 4;
    void *q8a[MAX_PARTS], *q8b[MAX_PARTS];  // Q8X scratch pairs of the decode parts
    uint64_t q8_blocks = 0;
    int32_t *d_tok, *d_pos, *d_slot, *d_next, *d_err;
    uint64_t slot_stride = 0, layer_stride = 0, v_off = 0;
    int32_t *h_io = nullptr;  // pinned staging: tok | pos | slot | next, R each
    std::map<std::tuple<int, int>, cudaGraphExec_t> graphs;
    bool use_graphs = true;
    bool use_fused_attention = true;
    bool split_decode = true;
    bool fuse_norm = true;   // RMSNorm + Q8 inside the QKV and gate/up GEMVs
    bool use_pdl = true;     // programmatic dependent launch between decode kernels
    bool no_prefill_tiles = false;  // SLM_PREFILL_ROWWISE=1: prefill through the per-row kernels
    int prefill_mode = SLM_PREFILL_EXACT;  // slm_model_set_prefill_mode
    bool gemm_tc = true;     // SLM_PREFILL_GEMM_EXACT=1: tensor-core prefill mode keeps exact projections
    int parts = 1;           // decode parts (streams) for batches of 16+ rows
    int pv_per_head = 1;     // softmax + PV per (row, query head): AttnArgs::pv_per_head
    bool pv_form_auto = true;  // SLM_PV_PER_HEAD unset: small decode steps take the cluster form
    bool shard_ffn = true;     // sharded prefill: Wo / FFN row-sharded (SLM_SHARD_FFN=0: replicated)
    int decode_mode = SLM_DECODE_EXACT;  // slm_model_set_decode_mode
    float *fd_part = nullptr;  // flash-decode partials [R][kvh][fd_nch][kv_mul*(hd+2)]
    int fd_nch = 0;
    cudaStream_t side[MAX_PARTS - 1] = {};  // streams of parts 1..
    cudaEvent_t ev_fork = nullptr, ev_join[MAX_PARTS - 1] = {};
    CUtensorMap vmap;        // V planes of the KV cache, for the fused attention
    CUtensorMap kmap;        // K planes, swizzled boxes for the scores kernel
    CUtensorMap vmap_half;   // V planes, boxes head_dim / 2 wide (split softmax + PV forms)
    bool have_vmap_half = false;
    CUtensorMap vmap_fine;   // V planes, V_FINE_POSITIONS-position boxes (fine-stage PV forms)
    bool have_vmap_fine = false;
    CUtensorMap kmap64;      // K planes, FD_ITEM_KEYS-key boxes for the flash-decode kernel
    bool have_kmap64 = false;
    // exact decode in one cluster launch: K planes with CL_BOX_KEYS-key boxes,
    // V planes with the box of cluster size 1, 2, 4, 8 (head_dim / C floats x
    // CL_BOX_KEYS * C positions)
    CUtensorMap kmap32, vmap_cl[4];
    bool have_kmap32 = false, have_vmap_cl[4] = {false, false, false, false};
    CUtensorMap amap;        // att scratch, probability tiles of the prefill softmax/PV
    bool have_vmap = false, have_kmap = false, have_amap = false;
    // KV-head-sharded batched prefill (slm_model_attach_shard)
    int shard_n = 1, shard_r = 0;
    ncclComm_t comm = nullptr;
    float *shard_send = nullptr, *shard_recv = nullptr;  // R*dim floats each
    // Communicator failures: every NCCL call and wait is bounded by
    // comm_timeout_ms; the first failure of a forward is kept here (code,
    // message) and returned by the entry point that ran the forward.
    uint32_t comm_timeout_ms = 120000;
    int comm_rc = SLM_OK;
    std::string comm_msg;
};

namespace {

// Drop the communicator after a failure (ncclCommAbort also ends any of its
// kernels still waiting for a peer); the model stays usable, the shard group
// does not (slm_model_prefill_batch then asks for a new attach).
void comm_abort(slm_model *m) {
    if (m->comm) nccl_api().abort(m->comm);
    m->comm = nullptr;
}

// Wait, bounded by the model's communicator timeout, until the non-blocking
// communicator has no operation in progress after a call that returned r.
int comm_settle(slm_model *m, ncclResult_t r, const char *what) {
    const NcclApi &api = nccl_api();
    const auto t0 = std::chrono::steady_clock::now();
    while (r == ncclInProgress) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(m->comm_timeout_ms)) {
            comm_abort(m);
            return fail(SLM_ERR_TIMEOUT, std::string(what) + ": no progress within the communicator timeout "
                                             "(a rank did not join); communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
        if (api.async_error(m->comm, &r) != ncclSuccess) break;
    }
    if (r != ncclSuccess) {
        const std::string msg = std::string(what) + ": " + api.error_string(r);
        comm_abort(m);
        return fail(SLM_ERR_CUDA, msg);
    }
    return SLM_OK;
}

// Wait for everything enqueued on the model stream when its work includes
// collectives: bounded by the communicator timeout, checking the
// communicator's asynchronous error meanwhile; on a timeout or an error the
// communicator is aborted (which ends its waiting kernels) before the stream
// is drained.
int comm_wait_stream(slm_model *m) {
    const NcclApi &api = nccl_api();
    cudaEvent_t ev = nullptr;
    CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    cudaEventRecord(ev, m->stream);
    const auto t0 = std::chrono::steady_clock::now();
    int rc = SLM_OK;
    for (;;) {
        const cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) {
            rc = fail(SLM_ERR_CUDA, std::string("collective step: ") + cudaGetErrorString(q));
            break;
        }
        ncclResult_t ar = ncclSuccess;
        if (m->comm && api.async_error(m->comm, &ar) == ncclSuccess && ar != ncclSuccess &&
            ar != ncclInProgress) {
            const std::string msg = std::string("collective step: ") + api.error_string(ar);
            comm_abort(m);
            rc = fail(SLM_ERR_CUDA, msg);
            break;
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(m->comm_timeout_ms)) {
            comm_abort(m);
            rc = fail(SLM_ERR_TIMEOUT, "collective step: not complete within the communicator timeout "
                                       "(a rank stopped taking part); communicator aborted");
            break;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    cudaStreamSynchronize(m->stream);
    cudaEventDestroy(ev);
    return rc;
}

// Upload a row-concatenation of Q4_0 matrices into wbuf at `*cursor`
// through the pinned staging path.
int upload_qmat(slm_model *m, Q4Uploader &up, const std::vector<std::pair<const void *, uint64_t>> &parts,
                uint64_t cols, uint64_t *cursor, QMat *out) {
    const uint64_t nb = cols / QK;
    uint64_t rows = 0;
    for (auto &p : parts) {
        if (!p.first) return fail(SLM_ERR_INVALID_ARG, "a weight tensor is null");
        if ((uintptr_t)p.first & 1) return fail(SLM_ERR_INVALID_ARG, "Q4_0 blocks must be 2-byte aligned");
        rows += p.second;
    }
    const uint64_t bytes = tiled_bytes(rows, cols);
    uint8_t *tiles = m->wbuf + *cursor;
    CUDA_TRY(cudaMemsetAsync(tiles, 0, bytes, up.stream()));  // rows past the last of the tile
    uint64_t row0 = 0;
    for (auto &p : parts) {
        TRY(up.rows(p.first, p.second, nb, row0, tiles));
        row0 += p.second;
    }
    out->tiles = tiles;
    out->rows = (int)rows;
    out->cols = (int)cols;
    *cursor += round_up(bytes, 256);
    return SLM_OK;
}

int upload_f32(slm_model *m, const float *src, uint64_t n, uint64_t *cursor, float **out) {
    CUDA_TRY(cudaMemcpy(m->wbuf + *cursor, src, n * 4, cudaMemcpyHostToDevice));
    *out = (float *)(m->wbuf + *cursor);
    *cursor += round_up(n * 4, 256);
    return SLM_OK;
}

Q8X q8view(void *p, uint64_t blocks) { return q8x_view(p, blocks); }
// The rows from row0 of a Q8X view with nb blocks per row.
Q8X q8rows(Q8X v, size_t row0, int nb) {
    const size_t b0 = row0 * (size_t)nb;
    v.qs += b0 * 32;
    v.c += b0 * 8;
    v.d += b0;
    return v;
}

// Records an event on the model stream at every phase boundary; the interval
// since the previous mark is attributed to the phase passed to mark().
struct Profiler {
    cudaStream_t st = nullptr;
    std::vector<cudaEvent_t> ev;
    std::vector<int> phase;
    size_t n = 0;
    void mark(int ph) {
        if (n < ev.size()) {
            cudaEventRecord(ev[n], st);
            phase[n] = ph;
            n++;
        }
    }
};

inline void mark(Profiler *p, int ph) {
    if (p) p->mark(ph);
}

// Enqueue one forward pass over the `n` activation rows [row0, row0+n),
// which already hold token ids / slots / positions in d_tok / d_slot / d_pos,
// on stream `st` with the Q8 scratch pair `part` (0 or 1).  Rows of
// different sequences are independent, so disjoint row ranges can run on
// different streams at the same time.
// Whether the QKV / gate-up GEMVs of an n-row step run the RMSNorm prologue
// themselves (staged weight tiles fit in shared memory); otherwise a separate
// RMSNorm + Q8 launch precedes them.  Activation rows are 16-byte aligned in
// the arena (dim is a multiple of 32), as the prologue's cp.async requires.
// From NORM_FUSE_MAX_ROWS rows up the prologue, which every weight-tile CTA
// repeats for its rows, costs more than one RMSNorm + Q8 launch over the rows
// (measured at 64 rows: 2.82 against 2.90 ms per config-3 decode step).
constexpr int NORM_FUSE_MAX_ROWS = 31;
bool qkv_norm_fused(const slm_model *m, int n) {
    return m->fuse_norm && n <= NORM_FUSE_MAX_ROWS &&
           gemv_fuses_norm((int)m->layers[0].wqkv.rows, (int)(m->cfg.dim / QK), EPI_QKV, n);
}
bool gate_up_norm_fused(const slm_model *m, int n) {
    return m->fuse_norm && n <= NORM_FUSE_MAX_ROWS &&
           gemv_fuses_norm(2 * (int)m->cfg.hidden_dim, (int)(m->cfg.dim / QK), EPI_SWIGLU_Q8, n);
}

// Decode attention of the exact mode in one cluster launch (SLM_PV_PER_HEAD
// 11): the cluster size for these rows, 0 when the form does not apply (the
// two-kernel forms run then).
int cl_map_index(int C) { return C == 1 ? 0 : C == 2 ? 1 : C == 4 ? 2 : 3; }
int decode_cluster(const slm_model *m, const AttnArgs &a) {
    const bool want = m->pv_per_head == 11 ||
                      (m->pv_form_auto && a.rows <= CLUSTER_AUTO_ROWS && attn_decode_cluster_preferred(a));
    if (!want || !m->have_kmap32) return 0;
    const int C = attn_decode_cluster_size(a);
    return C > 0 && m->have_vmap_cl[cl_map_index(C)] ? C : 0;
}

void enqueue_forward(slm_model *m, int row0, int n, int max_len, StepKind kind, cudaStream_t st,
                     int part, Profiler *prof = nullptr, int seq_rows = 0) {
    const slm_config &c = m->cfg;
    const int d = (int)c.dim, h = (int)c.hidden_dim;
    const size_t r0 = (size_t)row0;
    float *x = m->x + r0 * d, *x_mid = m->x_mid + r0 * d, *xb = m->xb + r0 * d;
    float *q = m->q + r0 * d;
    int32_t *tok = m->d_tok + r0, *pos = m->d_pos + r0, *slot = m->d_slot + r0;
    int32_t *next = m->d_next + r0;
    float *att = m->att + r0 * c.num_heads * c.max_seq_len;
    float *logits = m->logits + r0 * m->vocab;
    mark(prof, -1);
    launch_embed(m->embd.tiles, d / QK, tok, m->vocab, x, d, n, m->d_err, st);
    mark(prof, SLM_PHASE_EMBED);

    QkvArgs qa{};
    qa.q = q;
    qa.ldq = d;
    qa.k_base = m->kv;
    qa.v_base = m->kv + m->v_off;
    qa.slot = slot;
    qa.pos = pos;
    qa.slot_stride = m->slot_stride;
    qa.dim = d;
    qa.kv_dim = m->kvd;
    qa.head_dim = m->hd;
    qa.max_seq = (int)c.max_seq_len;
    qa.rope_cos = m->rope_cos;
    qa.rope_sin = m->rope_sin;
    qa.err = m->d_err;

    AttnArgs aa = attn_args_for(&c);
    aa.q = q;
    aa.ldq = d;
    aa.k_base = m->kv;
    aa.v_base = m->kv + m->v_off;
    aa.slot = slot;
    aa.pos = pos;
    aa.slot_stride = m->slot_stride;
    aa.att = att;
    aa.att_ld = c.max_seq_len;
    aa.out = xb;
    aa.ldo = d;
    aa.rows = n;
    aa.max_len = max_len;
    aa.err = m->d_err;
    aa.z_slot = 2LL * m->L;  // planes [slot][layer][K|V] from the first V plane
    aa.pdl = m->use_pdl;
    aa.tmax = row0 == 0 ? m->tmax : nullptr;
    aa.pv_per_head = m->pv_per_head;
    aa.fd_part = m->fd_part + r0 * c.num_kv_heads * (size_t)m->fd_nch * (c.num_heads / c.num_kv_heads) * (m->hd + 2);
    aa.fd_nch = m->fd_nch;
    aa.tmax_ld = m->tmax_ld;

    Q8X qa8 = q8view(m->q8a[part], m->q8_blocks), qb8 = q8view(m->q8b[part], m->q8_blocks);
    const bool fused = m->use_fused_attention && m->have_vmap && attention_fused_ok(aa);
    const int kv_mul = (int)(c.num_heads / c.num_kv_heads);
    // a batched prefill on a sharded model computes only this rank's
    // (sequence, KV head) units, then all-gathers the outputs before Wo
    const bool sharded = kind == STEP_PREFILL_BATCH && m->shard_n > 1 && fused;
    // ... and its Wo, RMSNorm and FFN row-sharded: this rank computes rows
    // [rs0, rs0 + ns) and one in-place all-gather of x per layer gives every
    // rank all rows for the next layer's QKV (rows are independent, so the
    // values are those of the unsharded step)
    const bool row_shard = sharded && m->shard_ffn && n % m->shard_n == 0;
    const int ns = row_shard ? n / m->shard_n : n, rs0 = row_shard ? m->shard_r * ns : 0;
    // prefill rows are runs of consecutive positions of one sequence
    aa.prefill_run = kind == STEP_PREFILL ? n : kind == STEP_PREFILL_BATCH ? seq_rows : 0;
    if (m->no_prefill_tiles) aa.prefill_run = 0;
    aa.prefill_tc = aa.prefill_run > 0 && m->prefill_mode == SLM_PREFILL_TENSOR_CORES;
    // the tensor-core prefill mode also runs the projections' int8 products on
    // the tensor cores (batches of 128+ rows)
    const bool gemm_tc = aa.prefill_tc && m->gemm_tc;
    if (kind == STEP_PREFILL_BATCH) {
        aa.rows_per_seq = seq_rows;
        aa.shard_n = sharded ? m->shard_n : 1;
        aa.shard_r = sharded ? m->shard_r : 0;
    }
    if (fused) {
        aa.write_probs = false;  // probabilities stay in shared memory
        if ((kv_mul * m->hd) % 32 == 0 && !sharded) aa.q8_out = qb8;
    }
    // decode rows in the opt-in split-K flash-decode mode (the Q8_0 of the
    // output inside the kernel)
    const bool flash = kind == STEP_DECODE && m->decode_mode == SLM_DECODE_FLASH && m->use_fused_attention &&
                       m->have_vmap && m->have_kmap64 && flash_decode_ok(aa);
    // decode rows of the exact mode: the one-launch cluster form when it applies
    const int ccl = kind == STEP_DECODE && fused && !flash ? decode_cluster(m, aa) : 0;
    const int n_units = kind == STEP_PREFILL_BATCH && seq_rows > 0 ? (n / seq_rows) * (int)c.num_kv_heads : 0;
    const bool norm_qkv = m->L > 0 && qkv_norm_fused(m, n);
    const bool norm_gu = m->L > 0 && gate_up_norm_fused(m, n);
    const float inv_d = 1.0f / (float)d;
    for (int l = 0; l < m->L; l++) {
        const LayerDev &ld = m->layers[l];
        // rmsnorm(x) -> Q8 (transformer.rs:411, kernels.rs:301), in the QKV
        // GEMV's prologue when it stages whole tiles
        GemvArgs g{};
        if (norm_qkv) {
            g.nx = x;
            g.ld_nx = d;
            g.nw = ld.rms_att;
            g.eps = c.rms_eps;
            g.inv_n = inv_d;
        } else {
            launch_rmsnorm_q8(x, d, ld.rms_att, d, c.rms_eps, nullptr, 0, qa8, n, st, m->use_pdl);
            mark(prof, SLM_PHASE_RMSNORM);
        }
        // Wq/Wk/Wv + RoPE + KV append (transformer.rs:413-428)
        g.w = ld.wqkv.tiles;
        g.rows = ld.wqkv.rows;
        g.nb = d / QK;
        g.x = qa8;
        g.batch = n;
        g.epi = EPI_QKV;
        qa.layer_off = (size_t)l * m->layer_stride;
        g.qkv = qa;
        g.err = m->d_err;
        g.pdl = m->use_pdl;
        g.tc = gemm_tc;
        launch_gemv(g, st);
        mark(prof, SLM_PHASE_QKV);
        // attention (transformer.rs:430-443)
        aa.layer_off = (size_t)l * m->layer_stride;
        aa.z_layer = 2LL * l;
        if (flash) {
            AttnArgs fa = aa;
            fa.q8_out = qb8;
            launch_flash_decode(fa, m->kmap64, m->vmap, st);
            mark(prof, SLM_PHASE_ATTN_FUSED);
        } else if (fused && ccl) {
            // scores, softmax, PV and the Q8_0 of the output in one cluster launch
            launch_attn_decode_cluster(aa, m->kmap32, m->vmap_cl[cl_map_index(ccl)], ccl, st);
            mark(prof, SLM_PHASE_ATTN_FUSED);
        } else if (fused) {
            // scores, then softmax + PV + the Q8_0 of the output
            launch_attn_fused(aa, m->vmap, m->have_kmap ? &m->kmap : nullptr,
                              m->have_amap && row0 == 0 ? &m->amap : nullptr, st,
                              m->have_vmap_half ? &m->vmap_half : nullptr,
                              m->have_vmap_fine ? &m->vmap_fine : nullptr);
            mark(prof, SLM_PHASE_ATTN_FUSED);
            if (sharded) {
                // this rank's units -> all ranks: one all-gather before Wo
                const int upr = n_units / m->shard_n, kd = kv_mul * m->hd;
                launch_shard_pack(xb, d, m->shard_send, upr, m->shard_n, m->shard_r,
                                  (int)c.num_kv_heads, kd, seq_rows, st);
                if (m->comm && m->comm_rc == SLM_OK) {
                    const ncclResult_t r = nccl_api().all_gather(
                        m->shard_send, m->shard_recv, (size_t)upr * seq_rows * kd, ncclFloat32, m->comm, st);
                    const int rc = comm_settle(m, r, "ncclAllGather");
                    if (rc != SLM_OK) {
                        m->comm_rc = rc;
                        m->comm_msg = g_err;
                    }
                }
                launch_shard_unpack(m->shard_recv, xb, d, upr, m->shard_n, (int)c.num_kv_heads, kd,
                                    seq_rows, st);
            }
            if (!aa.q8_out.qs) {
                launch_quantize_q8x(xb + (size_t)rs0 * d, d, d, q8rows(qb8, rs0, d / QK), ns, st);
                mark(prof, SLM_PHASE_QUANTIZE);
            }
        } else {
            launch_attn_scores(aa, st);
            mark(prof, SLM_PHASE_ATTN_SCORES);
            launch_attn_softmax(aa, st);
            mark(prof, SLM_PHASE_ATTN_SOFTMAX);
            launch_attn_pv(aa, st);
            mark(prof, SLM_PHASE_ATTN_PV);
            launch_quantize_q8x(xb, d, d, qb8, n, st);
            mark(prof, SLM_PHASE_QUANTIZE);
        }
        // Wo + residual (transformer.rs:445-446), this rank's rows when
        // row-sharded (rs0 = 0, ns = n otherwise)
        const size_t ro = (size_t)rs0 * d;
        g = GemvArgs{};
        g.w = ld.wo.tiles;
        g.rows = d;
        g.nb = d / QK;
        g.x = q8rows(qb8, rs0, d / QK);
        g.batch = ns;
        g.epi = EPI_RESIDUAL;
        g.out = x_mid + ro;
        g.ld_out = d;
        g.res = x + ro;
        g.ld_res = d;
        g.err = m->d_err;
        g.pdl = m->use_pdl;
        g.tc = gemm_tc;
        g.tc_any_batch = row_shard && n >= 128;
        launch_gemv(g, st);
        mark(prof, SLM_PHASE_WO);
        // rmsnorm(x_mid) -> gate/up -> SwiGLU -> Q8 (transformer.rs:448-475)
        g = GemvArgs{};
        if (norm_gu) {
            g.nx = x_mid + ro;
            g.ld_nx = d;
            g.nw = ld.rms_ffn;
            g.eps = c.rms_eps;
            g.inv_n = inv_d;
        } else {
            launch_rmsnorm_q8(x_mid + ro, d, ld.rms_ffn, d, c.rms_eps, nullptr, 0, q8rows(qa8, rs0, d / QK), ns, st,
                              m->use_pdl);
            mark(prof, SLM_PHASE_RMSNORM);
        }
        g.w = ld.wgu.tiles;
        g.rows = 2 * h;
        g.nb = d / QK;
        g.x = q8rows(qa8, rs0, d / QK);
        g.batch = ns;
        g.epi = EPI_SWIGLU_Q8;
        g.q8_out = q8rows(qb8, rs0, h / QK);
        g.err = m->d_err;
        g.pdl = m->use_pdl;
        g.tc = gemm_tc;
        g.tc_any_batch = row_shard && n >= 128;
        launch_gemv(g, st);
        mark(prof, SLM_PHASE_GATE_UP);
        // down + residual (transformer.rs:477-486)
        g = GemvArgs{};
        g.w = ld.wdown.tiles;
        g.rows = d;
        g.nb = h / QK;
        g.x = q8rows(qb8, rs0, h / QK);
        g.batch = ns;
        g.epi = EPI_RESIDUAL;
        g.out = x + ro;
        g.ld_out = d;
        g.res = x_mid + ro;
        g.ld_res = d;
        g.err = m->d_err;
        g.pdl = m->use_pdl;
        g.tc = gemm_tc;
        g.tc_any_batch = row_shard && n >= 128;
        launch_gemv(g, st);
        mark(prof, SLM_PHASE_DOWN);
        if (row_shard && m->comm && m->comm_rc == SLM_OK) {
            // every rank's rows of x to every rank (in place: this rank's rows
            // are already at their offset in x)
            const ncclResult_t r = nccl_api().all_gather(x + ro, x, (size_t)ns * d, ncclFloat32, m->comm, st);
            const int rc = comm_settle(m, r, "ncclAllGather");
            if (rc != SLM_OK) {
                m->comm_rc = rc;
                m->comm_msg = g_err;
            }
        }
    }
    if (kind == STEP_EMBED) return;
    // final RMSNorm + lm_head + argmax (transformer.rs:776-794 / 835-853)
    // prefill: the last row (of each sequence, for a batched prefill)
    const float *xs = kind == STEP_PREFILL ? x + (size_t)(n - 1) * d
                      : kind == STEP_PREFILL_BATCH ? x + (size_t)(seq_rows - 1) * d
                                                    : x;
    const size_t ldxs = kind == STEP_PREFILL_BATCH ? (size_t)seq_rows * d : (size_t)d;
    int rows = kind == STEP_PREFILL ? 1 : kind == STEP_PREFILL_BATCH ? n / seq_rows : n;
    launch_rmsnorm_q8(xs, ldxs, m->out_norm, d, c.rms_eps, nullptr, 0, qa8, rows, st);
    mark(prof, SLM_PHASE_RMSNORM);
    GemvArgs g{};
    g.w = m->lm_head.tiles;
    g.rows = m->vocab;
    g.nb = d / QK;
    g.x = qa8;
    g.batch = rows;
    g.epi = EPI_STORE;
    g.out = logits;
    g.ld_out = m->vocab;
    g.err = m->d_err;
    launch_gemv(g, st);
    mark(prof, SLM_PHASE_LM_HEAD);
    launch_argmax(logits, m->vocab, m->vocab, next, rows, st);
    mark(prof, SLM_PHASE_ARGMAX);
}

// kernel launches of one n-row decode part (enqueue_forward): embed; per
// layer: [rmsnorm], qkv, attention (fused: scores + softmax/PV, + quantize
// unless fused into it; or scores, softmax, pv, quantize), wo, [rmsnorm],
// gate/up, down; final rmsnorm, lm_head, argmax
// The attention arguments of a decode step that decide which kernels run.
AttnArgs decode_probe(const slm_model *m, int max_len) {
    AttnArgs a = attn_args_for(&m->cfg);
    a.ldq = m->cfg.dim;
    a.k_base = m->kv;
    a.v_base = m->kv + m->v_off;
    a.att = m->att;
    a.slot_stride = m->slot_stride;
    a.max_len = max_len;
    a.fd_part = m->fd_part;
    a.fd_nch = m->fd_nch;
    return a;
}

uint32_t decode_launches(const slm_model *m, int n) {
    const AttnArgs pa = decode_probe(m, (int)m->cfg.max_seq_len);
    const int kv_mul = (int)(m->cfg.num_heads / m->cfg.num_kv_heads);
    uint32_t attn = 4;  // scores, softmax, pv, quantize
    if (m->use_fused_attention && m->have_vmap && m->decode_mode == SLM_DECODE_FLASH && m->have_kmap64 &&
        flash_decode_ok(pa)) {
        AttnArgs pr = pa;
        pr.rows = n;
        attn = (uint32_t)flash_decode_launches(pr);  // splits (+ the combine, with the Q8_0 of the output)
    } else if (m->use_fused_attention && m->have_vmap && attention_fused_ok(pa)) {
        AttnArgs pr = pa;
        pr.rows = n;
        if (decode_cluster(m, pr))
            attn = 1;
        else if ((m->pv_per_head == 6 || m->pv_per_head == 7) && m->have_vmap_half && kv_mul <= 4 && (m->hd == 64 || m->hd == 128) &&
            kv_mul * m->hd / 2 <= 480)
            attn = 2;
        else if (m->pv_per_head >= 3 && m->pv_per_head <= 5 && kv_mul <= 4 && kv_mul * m->hd <= 480)
            attn = ((kv_mul * m->hd) % 32 == 0) ? 2 : 3;
        else if (m->pv_per_head)
            attn = (m->hd % 32 == 0) ? 2 : 3;
        else
            attn = ((kv_mul * m->hd) % 32 == 0) ? 2 : 3;
    }
    uint32_t per_layer = 4u + attn;
    if (m->L > 0 && !qkv_norm_fused(m, n)) per_layer++;
    if (m->L > 0 && !gate_up_norm_fused(m, n)) per_layer++;
    return 1u + per_layer * (uint32_t)m->L + 3u;
}

// Decode rows split into parts on parallel streams when the batch is large
// enough (8+ rows per part) for the parts to fill each other's latency gaps.
int decode_parts(const slm_model *m, int n) {
    if (!m->split_decode || n < 16) return 1;
    return std::max(1, std::min(m->parts, n / 8));
}

int len_bucket(const slm_model *m, int max_len) {
    int b = (max_len + 255) / 256 * 256;
    return std::min<int>(b, (int)m->cfg.max_seq_len);
}

// Enqueue a decode step of rows [0, n) (and the greedy advance): with P
// parts, rows [p*n/P, (p+1)*n/P) run on part p's stream (part 0 on the model
// stream), forked and joined with events so that a graph capture records P
// parallel branches.
void enqueue_decode(slm_model *m, int n, int bucket, bool advance) {
    const int parts = decode_parts(m, n);
    if (parts == 1) {
        enqueue_forward(m, 0, n, bucket, STEP_DECODE, m->stream, 0);
    } else {
        cudaEventRecord(m->ev_fork, m->stream);
        for (int p = 1; p < parts; p++) cudaStreamWaitEvent(m->side[p - 1], m->ev_fork, 0);
        for (int p = 0; p < parts; p++) {
            const int r0 = p * n / parts, r1 = (p + 1) * n / parts;
            enqueue_forward(m, r0, r1 - r0, bucket, STEP_DECODE, p ? m->side[p - 1] : m->stream, p);
        }
        for (int p = 1; p < parts; p++) {
            cudaEventRecord(m->ev_join[p - 1], m->side[p - 1]);
            cudaStreamWaitEvent(m->stream, m->ev_join[p - 1], 0);
        }
    }
    if (advance) launch_advance(m->d_tok, m->d_pos, m->d_next, n, m->stream);
}

// Run a decode step (optionally followed by the greedy advance) through a
// cached CUDA graph keyed by (rows, length bucket, advance).
int run_decode(slm_model *m, int n, int max_len, bool advance) {
    int bucket = len_bucket(m, max_len);
    if (!m->use_graphs) {
        enqueue_decode(m, n, bucket, advance);
        return launch_check("decode step");
    }
    auto key = std::make_tuple(n * 2 + (advance ? 1 : 0), bucket);
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaGraph_t graph = nullptr;
        CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        enqueue_decode(m, n, bucket, advance);
        cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(SLM_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
        }
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail(SLM_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
        it = m->graphs.emplace(key, exec).first;
    }
    CUDA_TRY(cudaGraphLaunch(it->second, m->stream));
    return SLM_OK;
}

int read_device_error(slm_model *m) {
    int32_t err = 0;
    CUDA_TRY(cudaMemcpyAsync(&err, m->d_err, 4, cudaMemcpyDeviceToHost, m->stream));
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    if (err) {
        CUDA_TRY(cudaMemsetAsync(m->d_err, 0, 4, m->stream));
        CUDA_TRY(cudaStreamSynchronize(m->stream));
        return fail(SLM_ERR_DEVICE_INPUT, err == 1   ? "token_id out of vocabulary bounds"
                                          : err == 2 ? "sequence position out of bounds"
                                                     : "a device wait timed out");
    }
    return SLM_OK;
}

int alloc_view(slm_model *m, uint64_t floats, float **out) {
    slm_slice s;
    TRY(slm_arena_alloc_slice(m->arena, floats, &s));
    *out = m->arena->base + s.offset;
    return SLM_OK;
}

}  // namespace

namespace {
void ensure_kernel_attributes() {
    // cudaFuncSetAttribute is per device and cheap; the attention softmax
    // stages up to max_seq_len floats in dynamic shared memory.
    static thread_local int done_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 31 && (done_mask & (1 << dev))) return;
    slm::set_attention_smem_limit(200 * 1024);
    slm::set_rmsnorm_smem_limit(200 * 1024);
    slm::set_gemv_smem_limit(200 * 1024);
    if (dev < 31) done_mask |= 1 << dev;
}
}  // namespace

SLM_EXPORT int slm_model_create(int device, const slm_config *cfg, const slm_model_weights *w,
                                uint32_t max_sequences, uint32_t max_rows, slm_model **out) {
    if (!out) return fail(SLM_ERR_INVALID_ARG, "out is null");
    *out = nullptr;
    TRY(check_config(cfg));
    if (!w || !w->token_embd || !w->output_norm || (!w->layers && w->num_layers))
        return fail(SLM_ERR_INVALID_ARG, "weights are null");
    if (w->vocab_size == 0) return fail(SLM_ERR_INVALID_ARG, "vocab_size must be positive");
    if (max_sequences == 0 || max_rows == 0)
        return fail(SLM_ERR_INVALID_ARG, "max_sequences and max_rows must be positive");
    for (uint32_t l = 0; l < w->num_layers; l++) {
        const slm_layer_weights &lw = w->layers[l];
        if (!lw.rms_att_weight || !lw.wq || !lw.wk || !lw.wv || !lw.wo || !lw.rms_ffn_weight ||
            !lw.w_gate || !lw.w_up || !lw.w_down)
            return fail(SLM_ERR_INVALID_ARG, "layer " + std::to_string(l) + " has a null tensor");
    }
    DeviceScope ds(device);
    ensure_kernel_attributes();
    slm_model *m = new slm_model();
    m->device = device;
    m->cfg = *cfg;
    m->L = (int)w->num_layers;
    m->vocab = (int)w->vocab_size;
    m->S = (int)max_sequences;
    m->R = (int)std::max(max_rows, max_sequences);
    m->hd = (int)(cfg->dim / cfg->num_heads);
    m->kvd = m->hd * (int)cfg->num_kv_heads;
    const uint64_t d = cfg->dim, h = cfg->hidden_dim, kvd = m->kvd, V = m->vocab;
    auto cleanup = [&](int rc) {
        slm_model_destroy(m);
        return rc;
    };
    cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    for (int p = 0; p + 1 < slm_model::MAX_PARTS && e == cudaSuccess; p++) {
        e = cudaStreamCreateWithFlags(&m->side[p], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->ev_join[p], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming);
    if (e != cudaSuccess) return cleanup(fail(SLM_ERR_CUDA, cudaGetErrorString(e)));

    // ---- weights: one device buffer
    uint64_t need = 0;
    auto add = [&](uint64_t rows, uint64_t cols) { need += round_up(tiled_bytes(rows, cols), 256); };
    for (int l = 0; l < m->L; l++) {
        add(d + 2 * kvd, d);
        add(d, d);
        add(2 * h, d);
        add(d, h);
        need += 2 * round_up(d * 4, 256);
    }
    add(V, d);
    add(V, d);
    need += round_up(d * 4, 256);
    e = cudaMalloc(&m->wbuf, need);
    if (e != cudaSuccess) return cleanup(fail(SLM_ERR_CUDA, std::string("weights: ") + cudaGetErrorString(e)));
    m->wbytes = need;
    uint64_t cur = 0;
    m->layers.resize(m->L);
    Q4Uploader up;
    int rc = up.begin();
    if (rc) return cleanup(rc);
    for (int l = 0; l < m->L; l++) {
        const slm_layer_weights &lw = w->layers[l];
        LayerDev &ld = m->layers[l];
        if ((rc = upload_qmat(m, up, {{lw.wq, d}, {lw.wk, kvd}, {lw.wv, kvd}}, d, &cur, &ld.wqkv)) ||
            (rc = upload_qmat(m, up, {{lw.wo, d}}, d, &cur, &ld.wo)) ||
            (rc = upload_qmat(m, up, {{lw.w_gate, h}, {lw.w_up, h}}, d, &cur, &ld.wgu)) ||
            (rc = upload_qmat(m, up, {{lw.w_down, d}}, h, &cur, &ld.wdown)) ||
            (rc = upload_f32(m, lw.rms_att_weight, d, &cur, &ld.rms_att)) ||
            (rc = upload_f32(m, lw.rms_ffn_weight, d, &cur, &ld.rms_ffn)))
            return cleanup(rc);
    }
    if ((rc = upload_qmat(m, up, {{w->token_embd, V}}, d, &cur, &m->embd)) ||
        (rc = upload_qmat(m, up, {{w->lm_head ? w->lm_head : w->token_embd, V}}, d, &cur,
                          &m->lm_head)) ||
        (rc = up.finish()) ||
        (rc = upload_f32(m, w->output_norm, d, &cur, &m->out_norm)))
        return cleanup(rc);

    // ---- arena (LayerWorkspace + BatchWorkspace + LayerKvCache per sequence)
    const uint64_t R = m->R, S = m->S, T = cfg->max_seq_len;
    const uint64_t maxk = std::max(d, h);
    m->q8_blocks = R * (maxk / QK);
    uint64_t q8f = (q8x_bytes(m->q8_blocks) + 3) / 4;
    m->v_off = T * kvd;
    m->layer_stride = 2 * T * kvd;
    m->slot_stride = (uint64_t)m->L * m->layer_stride;
    uint64_t a16 = ARENA_ALIGN_F32;
    uint64_t cap = 0;
    auto add_f = [&](uint64_t n) { cap = round_up(cap, a16) + n; };
    add_f(T * (m->hd / 2));  // rope cos
    add_f(T * (m->hd / 2));  // rope sin
    for (int i = 0; i < 4; i++) add_f(R * d);  // x, x_mid, xb, q
    add_f(R * d);                              // ybuf (embedding rows)
    add_f(d);                                  // embedding accumulator
    add_f(S * V);                              // logits
    add_f(R * cfg->num_heads * T);             // att
    m->tmax_ld = (int)((T + 31) / 32);
    add_f(R * cfg->num_heads * (uint64_t)m->tmax_ld);  // score maxima
    for (int i = 0; i < 2 * slm_model::MAX_PARTS; i++) add_f(q8f);  // Q8X pair per decode part
    m->fd_nch = flash_decode_chunks((int)T);
    const uint64_t kvm = cfg->num_heads / cfg->num_kv_heads;
    const uint64_t fd_floats = R * cfg->num_kv_heads * (uint64_t)m->fd_nch * kvm * (m->hd + 2);
    add_f(fd_floats);                          // flash-decode partials
    for (int i = 0; i < 5; i++) add_f(R);      // tok, pos, slot, next, err (int32)
    add_f(S * m->slot_stride);                 // KV
    rc = slm_arena_create(device, cap + a16, &m->arena);
    if (rc) return cleanup(rc);
    float *p;
    std::vector<float> cs(T * (m->hd / 2)), sn(T * (m->hd / 2));
    slm_rope_tables((uint32_t)T, (uint32_t)m->hd, cs.data(), sn.data());
    if ((rc = alloc_view(m, T * (m->hd / 2), &m->rope_cos)) ||
        (rc = alloc_view(m, T * (m->hd / 2), &m->rope_sin)) || (rc = alloc_view(m, R * d, &m->x)) ||
        (rc = alloc_view(m, R * d, &m->x_mid)) || (rc = alloc_view(m, R * d, &m->xb)) ||
        (rc = alloc_view(m, R * d, &m->q)) || (rc = alloc_view(m, R * d, &m->ybuf)) ||
        (rc = alloc_view(m, d, &m->emb)) || (rc = alloc_view(m, S * V, &m->logits)) ||
        (rc = alloc_view(m, R * cfg->num_heads * T, &m->att)) ||
        (rc = alloc_view(m, R * cfg->num_heads * (uint64_t)m->tmax_ld, &m->tmax)))
        return cleanup(rc);
    for (int i = 0; i < slm_model::MAX_PARTS; i++) {
        if ((rc = alloc_view(m, q8f, &p))) return cleanup(rc);
        m->q8a[i] = p;
        if ((rc = alloc_view(m, q8f, &p))) return cleanup(rc);
        m->q8b[i] = p;
    }
    if ((rc = alloc_view(m, fd_floats, &m->fd_part))) return cleanup(rc);
    int32_t **ints[] = {&m->d_tok, &m->d_pos, &m->d_slot, &m->d_next, &m->d_err};
    for (auto ip : ints) {
        if ((rc = alloc_view(m, R, &p))) return cleanup(rc);
        *ip = (int32_t *)p;
    }
    if ((rc = alloc_view(m, S * m->slot_stride, &m->kv))) return cleanup(rc);
    e = cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMallocHost(&m->h_io, 4 * R * sizeof(int32_t));
    if (e != cudaSuccess) return cleanup(fail(SLM_ERR_CUDA, cudaGetErrorString(e)));
    const char *env = getenv("SLM_DISABLE_GRAPHS");
    m->use_graphs = !(env && env[0] == '1');
    env = getenv("SLM_ATTENTION_3PASS");
    m->use_fused_attention = !(env && env[0] == '1');
    env = getenv("SLM_DECODE_ONE_STREAM");
    m->split_decode = !(env && env[0] == '1');
    m->pv_per_head = env_pv_per_head();
    m->pv_form_auto = env_pv_form_auto();
    env = getenv("SLM_SHARD_FFN");
    m->shard_ffn = !(env && env[0] == '0');
    env = getenv("SLM_DECODE_PARTS");
    if (env && env[0] >= '1' && env[0] <= '0' + slm_model::MAX_PARTS) m->parts = env[0] - '0';
    env = getenv("SLM_PREFILL_GEMM_EXACT");
    m->gemm_tc = !(env && env[0] == '1');
    env = getenv("SLM_PREFILL_ROWWISE");
    m->no_prefill_tiles = env && env[0] == '1';
    env = getenv("SLM_NO_PDL");
    m->use_pdl = !(env && env[0] == '1');
    env = getenv("SLM_UNFUSED_NORM");
    m->fuse_norm = !(env && env[0] == '1');
    // every V plane of the cache, addressed from the first one: plane
    // (slot, layer) sits at z = slot*2L + 2*layer, the last at S*2L - 2
    m->have_vmap = encode_v_map(&m->vmap, m->kv + m->v_off, m->kvd, (int)cfg->max_seq_len,
                                (uint64_t)S * 2 * m->L - 1, m->hd);
    m->have_vmap_half = m->hd % 2 == 0 && encode_v_map(&m->vmap_half, m->kv + m->v_off, m->kvd, (int)cfg->max_seq_len,
                                (uint64_t)S * 2 * m->L - 1, m->hd / 2);
    m->have_vmap_fine = encode_v_map(&m->vmap_fine, m->kv + m->v_off, m->kvd, (int)cfg->max_seq_len,
                                     (uint64_t)S * 2 * m->L - 1, m->hd, V_FINE_POSITIONS);
    // K plane (slot, layer) at z = slot*2L + 2*layer from the cache start
    m->have_kmap = encode_k_map(&m->kmap, m->kv, m->kvd, (int)cfg->max_seq_len,
                                (uint64_t)S * 2 * m->L - 1, m->hd);
    m->have_kmap64 = encode_k_map(&m->kmap64, m->kv, m->kvd, (int)cfg->max_seq_len,
                                (uint64_t)S * 2 * m->L - 1, m->hd, FD_ITEM_KEYS);
    m->have_kmap32 = encode_k_map(&m->kmap32, m->kv, m->kvd, (int)cfg->max_seq_len,
                                  (uint64_t)S * 2 * m->L - 1, m->hd, CL_BOX_KEYS);
    for (int i = 0; i < 4; i++)
        m->have_vmap_cl[i] = m->hd % (4 << i) == 0 &&
                             encode_v_map(&m->vmap_cl[i], m->kv + m->v_off, m->kvd, (int)cfg->max_seq_len,
                                          (uint64_t)S * 2 * m->L - 1, m->hd >> i, CL_BOX_KEYS << i);
    m->have_amap = encode_att_map(&m->amap, m->att, (int)cfg->max_seq_len, (int)cfg->num_heads,
                                  (uint64_t)R, (int)(cfg->num_heads / cfg->num_kv_heads));
    *out = m;
    return SLM_OK;
}

SLM_EXPORT void slm_model_destroy(slm_model *m) {
    if (!m) return;
    DeviceScope ds(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto st : m->side)
        if (st) cudaStreamSynchronize(st);
    for (auto &kv : m->graphs) cudaGraphExecDestroy(kv.second);
    if (m->ev_fork) cudaEventDestroy(m->ev_fork);
    for (auto ev : m->ev_join)
        if (ev) cudaEventDestroy(ev);
    for (auto st : m->side)
        if (st) cudaStreamDestroy(st);
    if (m->comm) nccl_api().destroy(m->comm);
    if (m->shard_send) cudaFree(m->shard_send);
    if (m->shard_recv) cudaFree(m->shard_recv);
    if (m->h_io) cudaFreeHost(m->h_io);
    if (m->arena) slm_arena_destroy(m->arena);
    if (m->wbuf) cudaFree(m->wbuf);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

SLM_EXPORT void *slm_model_stream(slm_model *m) { return m ? (void *)m->stream : nullptr; }

SLM_EXPORT uint64_t slm_model_device_bytes(const slm_model *m) {
    return m ? m->wbytes + m->arena->capacity * 4 : 0;
}

namespace {

// Stage host rows (token, slot, position) into the device row arrays.
int stage_rows(slm_model *m, int n, const int32_t *tok, const uint32_t *slot, uint32_t slot_const,
               const uint32_t *pos, uint32_t pos0) {
    int32_t *ht = m->h_io, *hp = m->h_io + m->R, *hs = m->h_io + 2 * m->R;
    for (int i = 0; i < n; i++) {
        ht[i] = tok[i];
        hs[i] = (int32_t)(slot ? slot[i] : slot_const);
        hp[i] = (int32_t)(pos ? pos[i] : pos0 + (uint32_t)i);
    }
    CUDA_TRY(cudaMemcpyAsync(m->d_tok, ht, n * 4, cudaMemcpyHostToDevice, m->stream));
    CUDA_TRY(cudaMemcpyAsync(m->d_pos, hp, n * 4, cudaMemcpyHostToDevice, m->stream));
    CUDA_TRY(cudaMemcpyAsync(m->d_slot, hs, n * 4, cudaMemcpyHostToDevice, m->stream));
    return SLM_OK;
}

int fetch_next(slm_model *m, int n, int32_t *next) {
    int32_t *hn = m->h_io + 3 * m->R;
    CUDA_TRY(cudaMemcpyAsync(hn, m->d_next, n * 4, cudaMemcpyDeviceToHost, m->stream));
    TRY(read_device_error(m));  // synchronizes
    std::memcpy(next, hn, n * 4);
    return SLM_OK;
}

int check_tokens(const slm_model *m, int n, const int32_t *tok) {
    for (int i = 0; i < n; i++)
        if (tok[i] < 0 || tok[i] >= m->vocab)
            return fail(SLM_ERR_OUT_OF_BOUNDS, "token_id out of vocabulary bounds");
    return SLM_OK;
}

}  // namespace

SLM_EXPORT int slm_model_decode_batch(slm_model *m, uint32_t n, const uint32_t *seqs,
                                      const int32_t *tokens, const uint32_t *pos,
                                      int32_t *next) {
    if (!m || !seqs || !tokens || !pos || !next) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (n == 0) return SLM_OK;
    if (n > (uint32_t)m->R || n > (uint32_t)m->S)
        return fail(SLM_ERR_CAPACITY, "batch larger than the model's max_rows/max_sequences");
    TRY(check_tokens(m, (int)n, tokens));
    uint32_t max_pos = 0;
    for (uint32_t i = 0; i < n; i++) {
        if (seqs[i] >= (uint32_t)m->S) return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence out of range");
        if (pos[i] >= m->cfg.max_seq_len)
            return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence position out of bounds");
        for (uint32_t k = 0; k < i; k++)
            if (seqs[k] == seqs[i]) return fail(SLM_ERR_INVALID_ARG, "duplicate sequence in batch");
        max_pos = std::max(max_pos, pos[i]);
    }
    DeviceScope ds(m->device);
    TRY(stage_rows(m, (int)n, tokens, seqs, 0, pos, 0));
    TRY(run_decode(m, (int)n, (int)max_pos + 1, false));
    return fetch_next(m, (int)n, next);
}

SLM_EXPORT int slm_model_forward_token(slm_model *m, uint32_t seq, int32_t token, uint32_t pos,
                                       int32_t *next) {
    return slm_model_decode_batch(m, 1, &seq, &token, &pos, next);
}

SLM_EXPORT int slm_model_prefill_tokens(slm_model *m, uint32_t seq, const int32_t *tokens,
                                        uint32_t n, uint32_t start_pos, int32_t *next) {
    if (!m || !tokens || !next) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (n == 0) return fail(SLM_ERR_INVALID_ARG, "prompt_tokens cannot be empty");
    if (n > (uint32_t)m->R) return fail(SLM_ERR_CAPACITY, "prompt longer than max_rows");
    if (seq >= (uint32_t)m->S) return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence out of range");
    if ((uint64_t)start_pos + n > m->cfg.max_seq_len)
        return fail(SLM_ERR_OUT_OF_BOUNDS, "start_pos + batch_size exceeds max_seq_len");
    TRY(check_tokens(m, (int)n, tokens));
    DeviceScope ds(m->device);
    TRY(stage_rows(m, (int)n, tokens, nullptr, seq, nullptr, start_pos));
    enqueue_forward(m, 0, (int)n, (int)(start_pos + n), STEP_PREFILL, m->stream, 0);
    TRY(launch_check("prefill"));
    return fetch_next(m, 1, next);
}

SLM_EXPORT int slm_model_prefill_batch(slm_model *m, uint32_t nseq, const uint32_t *seqs,
                                       const int32_t *tokens, uint32_t n, int32_t *next) {
    if (!m || !seqs || !tokens || !next) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (nseq == 0 || n == 0) return fail(SLM_ERR_INVALID_ARG, "empty batch or prompt");
    if ((uint64_t)nseq * n > (uint64_t)m->R || nseq > (uint32_t)m->S)
        return fail(SLM_ERR_CAPACITY, "nseq * n above max_rows or nseq above max_sequences");
    if (n > m->cfg.max_seq_len) return fail(SLM_ERR_OUT_OF_BOUNDS, "prompt longer than max_seq_len");
    for (uint32_t i = 0; i < nseq; i++)
        if (seqs[i] >= (uint32_t)m->S) return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence out of range");
    const int rows = (int)(nseq * n);
    TRY(check_tokens(m, rows, tokens));
    if (m->shard_n > 1) {
        if (!m->comm)
            return fail(SLM_ERR_INVALID_ARG, "the shard group failed earlier (communicator aborted); "
                                             "call slm_model_attach_shard again");
        if ((nseq * m->cfg.num_kv_heads) % (uint32_t)m->shard_n)
            return fail(SLM_ERR_SHAPE, "nseq * num_kv_heads must divide by the number of ranks");
        AttnArgs probe = attn_args_for(&m->cfg);
        probe.k_base = m->kv;
        probe.v_base = m->kv + m->v_off;
        probe.att = m->att;
        probe.slot_stride = m->slot_stride;
        probe.max_len = (int)n;
        if (!(m->use_fused_attention && m->have_vmap && attention_fused_ok(probe)))
            return fail(SLM_ERR_SHAPE, "sharded prefill needs the fused attention path");
    }
    DeviceScope ds(m->device);
    std::vector<uint32_t> slot(rows), pos(rows);
    for (int r = 0; r < rows; r++) {
        slot[r] = seqs[r / n];
        pos[r] = (uint32_t)(r % n);
    }
    TRY(stage_rows(m, rows, tokens, slot.data(), 0, pos.data(), 0));
    m->comm_rc = SLM_OK;
    enqueue_forward(m, 0, rows, (int)n, STEP_PREFILL_BATCH, m->stream, 0, nullptr, (int)n);
    TRY(launch_check("batched prefill"));
    if (m->shard_n > 1) {
        // the collectives make this forward wait on the other ranks: bounded
        const int rc = comm_wait_stream(m);
        if (m->comm_rc != SLM_OK) return fail(m->comm_rc, m->comm_msg);
        TRY(rc);
    }
    return fetch_next(m, (int)nseq, next);
}

SLM_EXPORT int slm_nccl_unique_id(void *id_out, uint64_t bytes) {
    if (!id_out || bytes != sizeof(ncclUniqueId))
        return fail(SLM_ERR_INVALID_ARG, "id buffer must hold " + std::to_string(sizeof(ncclUniqueId)) + " bytes");
    const NcclApi &api = nccl_api();
    if (!api.ok()) return fail(SLM_ERR_CUDA, "no NCCL library (libnccl.so.2) could be loaded");
    ncclUniqueId id;
    const ncclResult_t r = api.get_id(&id);
    if (r != ncclSuccess) return fail(SLM_ERR_CUDA, std::string("ncclGetUniqueId: ") + api.error_string(r));
    std::memcpy(id_out, &id, sizeof(id));
    return SLM_OK;
}

SLM_EXPORT int slm_model_set_prefill_mode(slm_model *m, int mode) {
    if (!m) return SLM_ERR_INVALID_ARG;
    if (mode != SLM_PREFILL_EXACT && mode != SLM_PREFILL_TENSOR_CORES) return SLM_ERR_INVALID_ARG;
    m->prefill_mode = mode;
    return SLM_OK;
}

SLM_EXPORT int slm_model_set_decode_mode(slm_model *m, int mode) {
    if (!m) return fail(SLM_ERR_INVALID_ARG, "model is null");
    if (mode != SLM_DECODE_EXACT && mode != SLM_DECODE_FLASH) return fail(SLM_ERR_INVALID_ARG, "unknown decode mode");
    if (mode == m->decode_mode) return SLM_OK;
    DeviceScope ds(m->device);
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    for (auto &kv : m->graphs) cudaGraphExecDestroy(kv.second);  // captured with the other kernels
    m->graphs.clear();
    m->decode_mode = mode;
    return SLM_OK;
}

SLM_EXPORT int slm_model_set_comm_timeout(slm_model *m, uint32_t timeout_ms) {
    if (!m || timeout_ms == 0) return fail(SLM_ERR_INVALID_ARG, "model is null or timeout is 0");
    m->comm_timeout_ms = timeout_ms;
    return SLM_OK;
}

SLM_EXPORT int slm_model_attach_shard(slm_model *m, const void *id, uint64_t bytes, int nranks,
                                      int rank) {
    if (!m) return fail(SLM_ERR_INVALID_ARG, "model is null");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(SLM_ERR_INVALID_ARG, "bad rank / nranks");
    if (m->comm) return fail(SLM_ERR_INVALID_ARG, "model already attached to a shard group");
    if (nranks == 1) {
        m->shard_n = 1;
        m->shard_r = 0;
        return SLM_OK;
    }
    if (!id || bytes != sizeof(ncclUniqueId)) return fail(SLM_ERR_INVALID_ARG, "bad NCCL unique id");
    const NcclApi &api = nccl_api();
    if (!api.ok()) return fail(SLM_ERR_CUDA, "no NCCL library (libnccl.so.2) could be loaded");
    DeviceScope ds(m->device);
    // the send/receive buffers are made once and kept across attach attempts
    const size_t bytes_buf = (size_t)m->R * m->cfg.dim * sizeof(float);
    if (!m->shard_send) CUDA_TRY(cudaMalloc(&m->shard_send, bytes_buf));
    if (!m->shard_recv) CUDA_TRY(cudaMalloc(&m->shard_recv, bytes_buf));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    // non-blocking set-up, so that a rank that never joins ends in a timeout
    // here instead of a wait without end
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = api.init_rank_config(&comm, nranks, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (comm) api.abort(comm);
        return fail(SLM_ERR_CUDA, std::string("ncclCommInitRankConfig: ") + api.error_string(r));
    }
    m->comm = comm;
    m->shard_n = 1;  // not sharded until the group is complete
    m->shard_r = 0;
    if (r == ncclInProgress) api.async_error(comm, &r);
    TRY(comm_settle(m, r, "ncclCommInitRankConfig"));
    m->shard_n = nranks;
    m->shard_r = rank;
    return SLM_OK;
}

SLM_EXPORT uint32_t slm_shard_units(uint32_t nseq, uint32_t num_kv_heads, uint32_t nranks,
                                    uint32_t rank, uint32_t *units_out, uint32_t capacity) {
    if (nranks == 0 || rank >= nranks || (nseq * num_kv_heads) % nranks) return 0;
    const uint32_t upr = nseq * num_kv_heads / nranks;
    for (uint32_t i = 0; i < upr && i < capacity; i++)
        if (units_out) units_out[i] = i * nranks + rank;
    return upr;
}

SLM_EXPORT int slm_model_generate(slm_model *m, uint32_t seq, const int32_t *prompt,
                                  uint32_t n_prompt, int32_t *out, uint32_t n_out, int32_t eos,
                                  uint32_t *generated) {
    if (!m || !generated) return fail(SLM_ERR_INVALID_ARG, "null argument");
    *generated = 0;
    if (n_out == 0 || n_prompt == 0) return SLM_OK;
    if (!prompt || !out) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (n_prompt > m->cfg.max_seq_len) return fail(SLM_ERR_OUT_OF_BOUNDS, "prompt longer than max_seq_len");
    int32_t next = 0;
    TRY(slm_model_prefill_tokens(m, seq, prompt, n_prompt, 0, &next));
    out[0] = next;
    uint32_t gen = 1;
    if (eos >= 0 && next == eos) {
        *generated = gen;
        return SLM_OK;
    }
    uint32_t pos = n_prompt;
    while (gen < n_out && pos < m->cfg.max_seq_len) {
        TRY(slm_model_forward_token(m, seq, next, pos, &next));
        out[gen++] = next;
        pos++;
        if (eos >= 0 && next == eos) break;
    }
    *generated = gen;
    return SLM_OK;
}

SLM_EXPORT int slm_model_embed_tokens(slm_model *m, uint32_t seq, const int32_t *tokens,
                                      uint32_t n, float *out_embedding) {
    if (!m || !tokens || !out_embedding) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (n == 0) return fail(SLM_ERR_INVALID_ARG, "tokens cannot be empty");
    if (n > (uint32_t)m->R || n > m->cfg.max_seq_len)
        return fail(SLM_ERR_CAPACITY, "too many tokens for max_rows/max_seq_len");
    if (seq >= (uint32_t)m->S) return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence out of range");
    TRY(check_tokens(m, (int)n, tokens));
    DeviceScope ds(m->device);
    const int d = (int)m->cfg.dim;
    TRY(stage_rows(m, (int)n, tokens, nullptr, seq, nullptr, 0));
    enqueue_forward(m, 0, (int)n, (int)n, STEP_EMBED, m->stream, 0);
    Q8X none{};
    launch_rmsnorm_q8(m->x, d, m->out_norm, d, m->cfg.rms_eps, m->ybuf, d, none, (int)n, m->stream);
    launch_mean_pool(m->ybuf, d, (int)n, d, 1.0f / (float)n, m->emb, m->stream);
    launch_l2norm_vec(m->emb, m->emb, d, m->cfg.rms_eps, m->stream);
    TRY(launch_check("embed"));
    std::vector<float> host(d);
    CUDA_TRY(cudaMemcpyAsync(host.data(), m->emb, d * 4, cudaMemcpyDeviceToHost, m->stream));
    TRY(read_device_error(m));
    std::memcpy(out_embedding, host.data(), d * 4);
    return SLM_OK;
}

SLM_EXPORT int slm_model_decode_steps_device(slm_model *m, uint32_t n, const uint32_t *seqs_dev,
                                             int32_t *tokens_dev, uint32_t *pos_dev,
                                             uint32_t steps, int32_t *out_dev,
                                             uint32_t max_pos_hint) {
    if (!m || !seqs_dev || !tokens_dev || !pos_dev) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (n == 0 || steps == 0) return SLM_OK;
    if (n > (uint32_t)m->R || n > (uint32_t)m->S)
        return fail(SLM_ERR_CAPACITY, "batch larger than the model's max_rows/max_sequences");
    if ((uint64_t)max_pos_hint + steps > m->cfg.max_seq_len)
        return fail(SLM_ERR_OUT_OF_BOUNDS, "decode would run past max_seq_len");
    DeviceScope ds(m->device);
    cudaStream_t st = m->stream;
    CUDA_TRY(cudaMemcpyAsync(m->d_slot, seqs_dev, n * 4, cudaMemcpyDeviceToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->d_tok, tokens_dev, n * 4, cudaMemcpyDeviceToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->d_pos, pos_dev, n * 4, cudaMemcpyDeviceToDevice, st));
    for (uint32_t s = 0; s < steps; s++) {
        TRY(run_decode(m, (int)n, (int)(max_pos_hint + s + 1), true));
        if (out_dev)
            CUDA_TRY(cudaMemcpyAsync(out_dev + (size_t)s * n, m->d_tok, n * 4,
                                     cudaMemcpyDeviceToDevice, st));
    }
    CUDA_TRY(cudaMemcpyAsync(tokens_dev, m->d_tok, n * 4, cudaMemcpyDeviceToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(pos_dev, m->d_pos, n * 4, cudaMemcpyDeviceToDevice, st));
    return SLM_OK;
}

namespace {
int kv_ptr(slm_model *m, uint32_t seq, uint32_t layer, uint32_t which, uint32_t row0,
           uint32_t nrows, float **p) {
    if (seq >= (uint32_t)m->S || layer >= (uint32_t)m->L || which > 1)
        return fail(SLM_ERR_OUT_OF_BOUNDS, "sequence/layer/which out of range");
    if ((uint64_t)row0 + nrows > m->cfg.max_seq_len)
        return fail(SLM_ERR_OUT_OF_BOUNDS, "rows beyond max_seq_len");
    *p = m->kv + seq * m->slot_stride + layer * m->layer_stride + which * m->v_off +
         (uint64_t)row0 * m->kvd;
    return SLM_OK;
}
}  // namespace

SLM_EXPORT int slm_model_kv_write(slm_model *m, uint32_t seq, uint32_t layer, uint32_t which,
                                  uint32_t row0, uint32_t nrows, const float *host) {
    if (!m || (!host && nrows)) return fail(SLM_ERR_INVALID_ARG, "null argument");
    float *p;
    TRY(kv_ptr(m, seq, layer, which, row0, nrows, &p));
    DeviceScope ds(m->device);
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    CUDA_TRY(cudaMemcpy(p, host, (size_t)nrows * m->kvd * 4, cudaMemcpyHostToDevice));
    return SLM_OK;
}

SLM_EXPORT int slm_model_kv_read(slm_model *m, uint32_t seq, uint32_t layer, uint32_t which,
                                 uint32_t row0, uint32_t nrows, float *host) {
    if (!m || (!host && nrows)) return fail(SLM_ERR_INVALID_ARG, "null argument");
    float *p;
    TRY(kv_ptr(m, seq, layer, which, row0, nrows, &p));
    DeviceScope ds(m->device);
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    CUDA_TRY(cudaMemcpy(host, p, (size_t)nrows * m->kvd * 4, cudaMemcpyDeviceToHost));
    return SLM_OK;
}

SLM_EXPORT int slm_model_read_logits(slm_model *m, uint32_t row, float *host) {
    if (!m || !host) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (row >= (uint32_t)m->S) return fail(SLM_ERR_OUT_OF_BOUNDS, "row out of range");
    DeviceScope ds(m->device);
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    CUDA_TRY(cudaMemcpy(host, m->logits + (size_t)row * m->vocab, (size_t)m->vocab * 4,
                        cudaMemcpyDeviceToHost));
    return SLM_OK;
}

SLM_EXPORT int slm_model_read_hidden(slm_model *m, uint32_t row, float *host) {
    if (!m || !host) return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (row >= (uint32_t)m->R) return fail(SLM_ERR_OUT_OF_BOUNDS, "row out of range");
    DeviceScope ds(m->device);
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    CUDA_TRY(cudaMemcpy(host, m->x + (size_t)row * m->cfg.dim, (size_t)m->cfg.dim * 4,
                        cudaMemcpyDeviceToHost));
    return SLM_OK;
}

SLM_EXPORT uint32_t slm_model_launches_per_decode_step(const slm_model *m, uint32_t n) {
    if (!m || n == 0) return 0;
    const int parts = decode_parts(m, (int)n);
    uint32_t total = 1u;  // the greedy advance
    for (int p = 0; p < parts; p++)
        total += decode_launches(m, (int)((p + 1) * n / parts - p * n / parts));
    return total;
}

SLM_EXPORT int slm_model_kv_write_device(slm_model *m, uint32_t seq, uint32_t layer,
                                         uint32_t which, uint32_t row0, uint32_t nrows,
                                         const float *src_dev) {
    if (!m || (!src_dev && nrows)) return fail(SLM_ERR_INVALID_ARG, "null argument");
    float *p;
    TRY(kv_ptr(m, seq, layer, which, row0, nrows, &p));
    DeviceScope ds(m->device);
    CUDA_TRY(cudaMemcpyAsync(p, src_dev, (size_t)nrows * m->kvd * 4, cudaMemcpyDeviceToDevice,
                             m->stream));
    return SLM_OK;
}

SLM_EXPORT int slm_model_profile_decode(slm_model *m, uint32_t n, const uint32_t *seqs_dev,
                                        int32_t *tokens_dev, uint32_t *pos_dev, uint32_t steps,
                                        uint32_t max_pos_hint, float *phase_ms) {
    if (!m || !seqs_dev || !tokens_dev || !pos_dev || !phase_ms)
        return fail(SLM_ERR_INVALID_ARG, "null argument");
    if (n == 0 || n > (uint32_t)m->R || n > (uint32_t)m->S)
        return fail(SLM_ERR_CAPACITY, "batch larger than the model's max_rows/max_sequences");
    if ((uint64_t)max_pos_hint + steps > m->cfg.max_seq_len)
        return fail(SLM_ERR_OUT_OF_BOUNDS, "decode would run past max_seq_len");
    DeviceScope ds(m->device);
    cudaStream_t st = m->stream;
    for (int i = 0; i < SLM_NUM_PHASES; i++) phase_ms[i] = 0.0f;
    Profiler prof;
    prof.st = st;
    size_t nev = 8 + (size_t)m->L * 12;
    prof.ev.resize(nev);
    prof.phase.resize(nev);
    for (auto &e : prof.ev) CUDA_TRY(cudaEventCreate(&e));
    int rc = SLM_OK;
    cudaError_t e = cudaMemcpyAsync(m->d_slot, seqs_dev, n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_tok, tokens_dev, n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_pos, pos_dev, n * 4, cudaMemcpyDeviceToDevice, st);
    for (uint32_t s = 0; s < steps && e == cudaSuccess && rc == SLM_OK; s++) {
        prof.n = 0;
        enqueue_forward(m, 0, (int)n, len_bucket(m, (int)(max_pos_hint + s + 1)), STEP_DECODE,
                        st, 0, &prof);
        launch_advance(m->d_tok, m->d_pos, m->d_next, (int)n, st);
        prof.mark(SLM_PHASE_ADVANCE);
        e = cudaStreamSynchronize(st);
        for (size_t i = 1; i < prof.n && e == cudaSuccess; i++) {
            float ms = 0.0f;
            e = cudaEventElapsedTime(&ms, prof.ev[i - 1], prof.ev[i]);
            if (prof.phase[i] >= 0 && prof.phase[i] < SLM_NUM_PHASES) phase_ms[prof.phase[i]] += ms;
        }
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(tokens_dev, m->d_tok, n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(pos_dev, m->d_pos, n * 4, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    for (auto &ev : prof.ev) cudaEventDestroy(ev);
    if (e != cudaSuccess) return fail(SLM_ERR_CUDA, std::string("profile: ") + cudaGetErrorString(e));
    return rc;
}
