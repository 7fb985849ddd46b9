/*
 * Forced-include shim for compiling the reference's CUDA operators (measurement
 * only: the reference's own GPU kernels timed on the same B200; Makefile target
 * `ref_cuda`).  On top of ref_shim.h (ops moved to `serron_ref::`), it supplies
 * the current CUDA stream that torch 2.11's stable accelerator API cannot hand
 * out (its Stream has no nativeHandle()): the build copies the reference sources
 * and points gpu/utils/launch.h's one use of it here.
 */
#ifndef SERRON_ORACLE_REF_CUDA_SHIM_H
#define SERRON_ORACLE_REF_CUDA_SHIM_H

#include "ref_shim.h"

#include <cstdint>

extern "C" int32_t aoti_torch_get_current_cuda_stream(int32_t device_index, void** ret_stream);

inline void* serron_ref_current_stream(int device_index) {
    void* stream = nullptr;
    aoti_torch_get_current_cuda_stream(device_index, &stream);
    return stream;
}

#endif
