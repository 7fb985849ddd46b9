// serron_backward_static_scratch: erosion / dilation backward that allocates nothing.
//
// The ordinary backward entry points take a device workspace from the caller (winner records and the
// grad_kernel partial sums).  Some callers cannot provide one: a host program binding the C ABI
// directly that owns only its input and output buffers and has no device allocator to size extra
// memory with, and callers that must not call cudaMalloc / cudaFree between launches, because those
// calls synchronise the device and can fail at any time under a fixed memory budget.  For them this
// entry point runs the same backward with its scratch in a fixed array of this library's own device
// memory, reserved when the library's module loads on a device, so no call ever allocates.
//
// Limits and rules of use
//   - the scratch holds SERRON_STATIC_SCRATCH_BYTES (32 MiB) per device; a call whose workspace would
//     be larger is rejected with SERRON_ERR_WORKSPACE before any work is enqueued;
//   - every call looks the array's address up (cudaGetSymbolAddress with that device current), so an
//     address never outlives the context it belongs to (a cudaDeviceReset between calls is fine); the
//     first call on a device may load the module for it: make that first call outside any stream capture;
//   - there is one array per device, so calls that can overlap on the GPU (on two streams, or from two
//     host threads on one device) race on it: order such calls on one stream or with events;
//   - nothing in the array has to start at zero: a call writes every scratch byte before reading it
//     (the forward pass writes all winner records, the grad_kernel kernel zeroes its own bins).
#include "serron_b200.h"

#include <cuda_runtime.h>

#include <sstream>
#include <string>

namespace serron {
void set_last_error(const std::string& message);  // api.cu: the message serron_last_error returns
}  // namespace serron

namespace {

constexpr int64_t kScratchBytes = SERRON_STATIC_SCRATCH_BYTES;
__device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Device address of g_scratch on `device`, looked up with that device current.  Only the failure of a
// call made here is cleared from the runtime's last-error slot; an error the caller left pending stays.
cudaError_t scratch_address(int device, void** out) {
    int previous = -1;
    if (cudaGetDevice(&previous) != cudaSuccess) {
        cudaGetLastError();
        previous = -1;
    }
    cudaError_t err = previous == device ? cudaSuccess : cudaSetDevice(device);
    void* address = nullptr;
    if (err == cudaSuccess) err = cudaGetSymbolAddress(&address, g_scratch);
    if (previous >= 0 && previous != device) cudaSetDevice(previous);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return err;
    }
    *out = address;
    return cudaSuccess;
}

}  // namespace

extern "C" int serron_backward_static_scratch(int32_t op, const void* grad_output, const int64_t* grad_output_sizes,
                                              int64_t grad_output_dim, const void* input, const int64_t* input_sizes,
                                              int64_t input_dim, const void* kernel, const int64_t* kernel_sizes,
                                              int64_t kernel_dim, int32_t dtype, int64_t border, int32_t flat,
                                              int32_t need_kernel_grad, int64_t algo, void* grad_input,
                                              void* grad_kernel, int32_t device, void* stream) {
    const char* name = "serron_backward_static_scratch";
    if (op != SERRON_ERODE && op != SERRON_DILATE) {
        serron::set_last_error(std::string(name) + ": invalid op " + std::to_string(op));
        return SERRON_ERR_INVALID;
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) {
        cudaGetLastError();
        count = 0;
    }
    if (device < 0 || device >= count) {
        serron::set_last_error(std::string(name) + ": invalid device " + std::to_string(device));
        return SERRON_ERR_INVALID;
    }
    void* scratch = nullptr;
    const cudaError_t err = scratch_address(device, &scratch);
    if (err != cudaSuccess) {
        serron::set_last_error(std::string(name) + ": cannot find the static scratch on device " +
                               std::to_string(device) + ": " + cudaGetErrorName(err));
        return SERRON_ERR_CUDA;
    }
    auto backward = op == SERRON_ERODE ? serron_erode_backward : serron_dilate_backward;
    const int rc = backward(grad_output, grad_output_sizes, grad_output_dim, input, input_sizes, input_dim, kernel,
                            kernel_sizes, kernel_dim, dtype, border, flat, need_kernel_grad, algo, grad_input,
                            grad_kernel, scratch, kScratchBytes, device, stream);
    if (rc == SERRON_ERR_WORKSPACE) {
        // the workspace check runs before any launch: nothing was enqueued
        std::ostringstream oss;
        oss << name << ": this call needs more scratch than the " << kScratchBytes
            << " bytes of the static array (" << serron_last_error()
            << "); use serron_erode_backward / serron_dilate_backward with a caller workspace";
        serron::set_last_error(oss.str());
    }
    return rc;
}
