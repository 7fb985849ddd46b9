// Measured min/max issue rate of this GPU: the compute roofline of the morphology kernels, whose inner
// work is compare-select (FP32 FMNMX, or packed half2 / bfloat162 min/max).  A separate library from the
// operators: it exists only to give the measurement a number.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

namespace {

constexpr int kChains = 8;     // independent dependency chains per thread
constexpr int kIters = 4096;   // loop trips; each does 2 min/max per chain

template <typename V>
__device__ __forceinline__ V vmin(V a, V b);
template <typename V>
__device__ __forceinline__ V vmax(V a, V b);
template <> __device__ __forceinline__ float vmin(float a, float b) { return fminf(a, b); }
template <> __device__ __forceinline__ float vmax(float a, float b) { return fmaxf(a, b); }
template <> __device__ __forceinline__ __half2 vmin(__half2 a, __half2 b) { return __hmin2(a, b); }
template <> __device__ __forceinline__ __half2 vmax(__half2 a, __half2 b) { return __hmax2(a, b); }
template <> __device__ __forceinline__ __nv_bfloat162 vmin(__nv_bfloat162 a, __nv_bfloat162 b) { return __hmin2(a, b); }
template <> __device__ __forceinline__ __nv_bfloat162 vmax(__nv_bfloat162 a, __nv_bfloat162 b) { return __hmax2(a, b); }

template <typename V>
__device__ __forceinline__ V from_float(float f);
template <> __device__ __forceinline__ float from_float(float f) { return f; }
template <> __device__ __forceinline__ __half2 from_float(float f) { return __float2half2_rn(f); }
template <> __device__ __forceinline__ __nv_bfloat162 from_float(float f) { return __float2bfloat162_rn(f); }

// Cross-coupled chains: a[c] = min(a[c], b[c]); b[c] = max(b[c], a[(c + 1) % kChains]).
template <typename V>
__global__ void __launch_bounds__(256) minmax_chain_kernel(const float* seed, V* sink) {
    V a[kChains], b[kChains];
    const float s = seed[threadIdx.x & 31];
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
        a[c] = from_float<V>(s + c);
        b[c] = from_float<V>(s - c);
    }
#pragma unroll 4
    for (int it = 0; it < kIters; ++it) {
#pragma unroll
        for (int c = 0; c < kChains; ++c) {
            a[c] = vmin<V>(a[c], b[c]);
            b[c] = vmax<V>(b[c], a[(c + 1) % kChains]);
        }
    }
    V acc = a[0];
#pragma unroll
    for (int c = 1; c < kChains; ++c) acc = vmin<V>(vmax<V>(acc, a[c]), b[c]);
    sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

template <typename V>
int measure(int device, double* lane_ops_per_s) {
    cudaSetDevice(device);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const int blocks = sms * 8, threads = 256;
    float* seed = nullptr;
    V* sink = nullptr;
    if (cudaMalloc(&seed, 32 * sizeof(float)) != cudaSuccess) return 1;
    if (cudaMalloc(&sink, size_t(blocks) * threads * sizeof(V)) != cudaSuccess) return 1;
    cudaMemset(seed, 0, 32 * sizeof(float));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    minmax_chain_kernel<V><<<blocks, threads>>>(seed, sink);  // warm-up
    cudaEventRecord(e0);
    const int reps = 5;
    for (int r = 0; r < reps; ++r) minmax_chain_kernel<V><<<blocks, threads>>>(seed, sink);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    const int err = static_cast<int>(cudaGetLastError());
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(seed);
    cudaFree(sink);
    if (err) return err;
    const double lanes = std::is_same<V, float>::value ? 1.0 : 2.0;
    const double ops = double(blocks) * threads * reps * kIters * kChains * 2 * lanes;
    *lane_ops_per_s = ops / (ms * 1e-3);
    return 0;
}

}  // namespace

// kind: 0 FP32 min/max, 1 half2, 2 bfloat162.  Writes element min/max operations per second (packed
// types count both lanes).  Returns 0 or a CUDA error code.
extern "C" __attribute__((visibility("default"))) int serron_measure_minmax_rate(int kind, int device,
                                                                                 double* lane_ops_per_s) {
    switch (kind) {
    case 0: return measure<float>(device, lane_ops_per_s);
    case 1: return measure<__half2>(device, lane_ops_per_s);
    case 2: return measure<__nv_bfloat162>(device, lane_ops_per_s);
    default: return -1;
    }
}
