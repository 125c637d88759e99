// Internal helpers shared by the host and device translation units of libtcc_spmm_b200.
#pragma once

#include "tcc_spmm_b200.h"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <exception>
#include <new>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace tcc {

// Thread-local message behind tcc_last_error().
void setLastError(const std::string& message);
void clearLastError();

// A CUDA failure, reported as TCC_CUDA_ERROR (the reference throws std::runtime_error).
struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
// A bounded device wait that ran out.
struct DeviceTimeout : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// Run `body` and translate any exception into a tcc_status plus message.
template <typename Body> int guarded(Body&& body) {
    try {
        clearLastError();
        body();
        return TCC_OK;
    } catch (const std::invalid_argument& e) {
        setLastError(e.what());
        return TCC_INVALID_ARGUMENT;
    } catch (const std::overflow_error& e) {
        setLastError(e.what());
        return TCC_OVERFLOW;
    } catch (const DeviceTimeout& e) {
        setLastError(e.what());
        return TCC_DEVICE_TIMEOUT;
    } catch (const CudaError& e) {
        setLastError(e.what());
        return TCC_CUDA_ERROR;
    } catch (const std::bad_alloc&) {
        setLastError("host allocation failed");
        return TCC_INTERNAL;
    } catch (const std::exception& e) {
        setLastError(e.what());
        return TCC_INTERNAL;
    } catch (...) {
        setLastError("unknown error");
        return TCC_INTERNAL;
    }
}

// Map a tcc_status back to the exception the reference API throws (C++ drop-in layer).
[[noreturn]] void throwStatus(int status, const char* message);
inline void check(int status) {
    if (status != TCC_OK)
        throwStatus(status, tcc_last_error());
}

// Static work split over host threads: body(begin, end) on contiguous blocks of [0, n).
// Blocks are taken dynamically; `grain` items per block.
template <typename Body>
void parallelFor(std::size_t n, std::size_t grain, unsigned threads, Body&& body) {
    if (n == 0)
        return;
    if (threads == 0)
        threads = std::max(1u, std::thread::hardware_concurrency());
    const std::size_t blocks = (n + grain - 1) / grain;
    threads = static_cast<unsigned>(std::min<std::size_t>(threads, blocks));
    if (threads <= 1) {
        body(std::size_t(0), n);
        return;
    }
    std::atomic<std::size_t> next{0};
    std::exception_ptr failure;
    std::atomic<bool> failed{false};
    auto worker = [&] {
        try {
            for (;;) {
                const std::size_t b = next.fetch_add(1);
                if (b >= blocks || failed.load())
                    break;
                body(b * grain, std::min(n, (b + 1) * grain));
            }
        } catch (...) {
            if (!failed.exchange(true))
                failure = std::current_exception();
        }
    };
    std::vector<std::thread> pool;
    pool.reserve(threads - 1);
    for (unsigned t = 1; t < threads; ++t)
        pool.emplace_back(worker);
    worker();
    for (auto& t : pool)
        t.join();
    if (failure)
        std::rethrow_exception(failure);
}

} // namespace tcc
