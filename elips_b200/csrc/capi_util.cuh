// Helpers shared by the C ABI translation units: exceptions from the engine
// become ELIPS_B200_* status codes, and host-pointer calls run on a stream of
// their own so concurrent callers never share one.
#pragma once

#include <cstdio>
#include <new>

#include "../../include/elips_b200.h"
#include "engine.cuh"

namespace eb {

template <class Fn>
int guarded(Fn&& fn) {
    try {
        fn();
        return ELIPS_B200_OK;
    } catch (const Error& e) {
        std::fprintf(stderr, "elips_b200: %s\n", e.what.c_str());
        return e.code;
    } catch (const std::bad_alloc&) {
        return ELIPS_B200_INSUFFICIENT_MEMORY;
    } catch (...) {
        return ELIPS_B200_KERNEL_LAUNCH_FAILED;
    }
}

struct OwnedStream {
    cudaStream_t s = nullptr;
    OwnedStream() {
        check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), ELIPS_B200_INITIALIZATION_FAILED,
                   "cudaStreamCreate");
    }
    ~OwnedStream() { cudaStreamDestroy(s); }
    OwnedStream(const OwnedStream&) = delete;
    OwnedStream& operator=(const OwnedStream&) = delete;
};

}  // namespace eb
