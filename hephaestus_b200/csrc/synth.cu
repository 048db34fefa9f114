// synth.cu — device generators of the seeded synthetic inputs (test and
// benchmark support; see include/heph/heph_synth.h).
#include "common.cuh"
#include "device_utils.cuh"
#include "heph/heph_synth.h"

namespace heph {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t hash(uint64_t seed, uint64_t i) { return splitmix64((seed << 32) ^ i); }

__global__ void fill_kernel(void *out, uint64_t count, int kind, uint64_t seed, uint64_t base) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride) {
        const uint64_t i = base + k;
        switch (kind) {
            case HEPH_SYNTH_F32_UNIFORM_PM1:
                static_cast<float *>(out)[k] = -1.0f + 2.0f * ((float)(hash(seed, i) >> 40) * 0x1p-24f);
                break;
            case HEPH_SYNTH_U32_LOW4:
                static_cast<uint32_t *>(out)[k] = (uint32_t)(hash(seed, i) & 15u);
                break;
            case HEPH_SYNTH_F32_NORMAL: {
                const double u1 = (double)((hash(seed, 2 * i) >> 11) + 1) * 0x1p-53;
                const double u2 = (double)(hash(seed, 2 * i + 1) >> 11) * 0x1p-53;
                static_cast<float *>(out)[k] = (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
                break;
            }
            case HEPH_SYNTH_F64_UNIT:
                static_cast<double *>(out)[k] = (double)(hash(seed, i) >> 11) * 0x1p-53;
                break;
            case HEPH_SYNTH_I32_PM1000:
                static_cast<int32_t *>(out)[k] = (int32_t)(hash(seed, i) % 2001u) - 1000;
                break;
        }
    }
}

// One warp per row: first argmax, then the seeded tie.
__global__ void ties_kernel(float *x, uint64_t rows, uint64_t cols, uint64_t seed) {
    const uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows || cols == 0) return;
    if (hash(seed, (1ull << 32) + row) % 100u != 0) return;
    float *r = x + row * cols;
    float best = r[lane < cols ? lane : 0];
    uint32_t bi = lane < cols ? lane : 0xffffffffu;
    for (uint64_t c = lane + 32; c < cols; c += 32)
        if (r[c] > best) {
            best = r[c];
            bi = (uint32_t)c;
        }
    warp_arg_fold<float, OP_MAX>(best, bi);
    if (lane == 0) {
        uint64_t j = hash(seed, (1ull << 33) + row) % cols;
        if (j == bi) j = (j + 1) % cols;
        r[j] = best;
    }
}

}  // namespace
}  // namespace heph

using namespace heph;

extern "C" heph_status heph_synth_fill(heph_device *device, heph_buffer *buffer, uint64_t offset,
                                       uint64_t count, heph_synth_kind kind, uint64_t seed,
                                       uint64_t index_base, heph_stream stream) {
    if (!device || !buffer) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    static const heph_dtype want[] = {HEPH_F32, HEPH_U32, HEPH_F32, HEPH_F64, HEPH_I32};
    if ((int)kind < 0 || (int)kind > 4) return fail(HEPH_INVALID_CONFIGURATION, "unknown generator");
    if (buffer->dtype != want[kind]) return fail(HEPH_INVALID_CONFIGURATION, "generator does not match the buffer type");
    if (offset > buffer->len || count > buffer->len - offset)
        return fail(HEPH_LENGTH_MISMATCH, "generated range exceeds the buffer");
    if (count == 0) return HEPH_OK;
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    char *p = static_cast<char *>(buffer->ptr) + offset * dtype_size(buffer->dtype);
    const unsigned grid = (unsigned)std::min<uint64_t>((count + 255) / 256, (uint64_t)device->sm_count * 16);
    fill_kernel<<<grid, 256, 0, resolve_stream(device, stream)>>>(p, count, (int)kind, seed, index_base);
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "generator launch");
    return HEPH_OK;
}

extern "C" heph_status heph_synth_inject_row_ties(heph_device *device, heph_buffer *matrix, uint64_t rows,
                                                  uint64_t cols, uint64_t seed, heph_stream stream) {
    if (!device || !matrix) return fail(HEPH_INVALID_CONFIGURATION, "null argument");
    if (matrix->dtype != HEPH_F32) return fail(HEPH_INVALID_CONFIGURATION, "ties are injected into f32 matrices");
    if (rows * cols > matrix->len) return fail(HEPH_LENGTH_MISMATCH, "matrix exceeds the buffer");
    if (rows == 0 || cols == 0) return HEPH_OK;
    heph_status st = bind(device);
    if (st != HEPH_OK) return st;
    const uint64_t blocks = (rows * 32 + 255) / 256;
    ties_kernel<<<(unsigned)blocks, 256, 0, resolve_stream(device, stream)>>>(
        static_cast<float *>(matrix->ptr), rows, cols, seed);
    HEPH_CUDA_TRY(cudaGetLastError(), HEPH_DISPATCH_FAILED, "tie injection launch");
    return HEPH_OK;
}
