/*
 * Forced-include shim for compiling the reference's CPU operators (test
 * infrastructure only, see Makefile target `ref`).
 *
 * 1. The reference registers its ops under `serron::`, which is also the
 *    namespace this project's own ops use.  Pre-including the reference's
 *    registration header (it has an include guard) and redefining the
 *    extension name moves the reference build to `serron_ref::`, so both
 *    libraries load side by side in one process.
 * 2. torch 2.11's HeaderOnlyArrayRef lacks operator==, which the reference's
 *    CPU backward uses to compare two size lists
 *    (packages/serron/csrc/cpu/morphology/backward.cpp:378).
 */
#ifndef SERRON_ORACLE_REF_SHIM_H
#define SERRON_ORACLE_REF_SHIM_H

#include <compat/registration.h>
#undef TORCH_EXTENSION_NAME
#define TORCH_EXTENSION_NAME serron_ref

#if __has_include(<torch/headeronly/util/HeaderOnlyArrayRef.h>)
#include <torch/headeronly/util/HeaderOnlyArrayRef.h>
#include <algorithm>
namespace c10 {
template <typename T>
inline bool operator==(HeaderOnlyArrayRef<T> a, HeaderOnlyArrayRef<T> b) {
    return a.size() == b.size() && std::equal(a.begin(), a.end(), b.begin());
}
} // namespace c10
#endif

#endif
