// abi.hpp — C ABI boundary helpers: status mapping, thread-local last error,
// host-side fault table.
#pragma once

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "common.cuh"

namespace faber {

inline thread_local std::string g_last_error;

inline FaberRtStatusV1 status(int code) { return FaberRtStatusV1{code}; }

// Host-side fault injection table (test support): entry name -> (status, remaining).
struct FaultTable {
  std::mutex mu;
  std::map<std::string, std::pair<int, unsigned>> table;
  int take(const char* entry) {
    std::lock_guard<std::mutex> lk(mu);
    auto it = table.find(entry);
    if (it == table.end() || it->second.second == 0) return 0;
    it->second.second -= 1;
    return it->second.first;
  }
};
inline FaultTable g_faults;

// Run `fn` and convert every failure into a status: Error -> its code,
// std::bad_alloc -> ALLOCATION, any other exception -> PANIC (the reference's
// catch_unwind -> STATUS_PANIC).
template <class F>
FaberRtStatusV1 guarded(const char* entry, F&& fn) {
  try {
    if (int injected = g_faults.take(entry)) {
      g_last_error = std::string(entry) + ": injected fault";
      return status(injected);
    }
    fn();
    return status(FABER_STATUS_OK);
  } catch (const Error& e) {
    g_last_error = std::string(entry) + ": " + e.what();
    return status(e.code);
  } catch (const std::bad_alloc&) {
    g_last_error = std::string(entry) + ": host allocation failed";
    return status(FABER_STATUS_ALLOCATION);
  } catch (const std::exception& e) {
    g_last_error = std::string(entry) + ": " + e.what();
    return status(FABER_STATUS_PANIC);
  } catch (...) {
    g_last_error = std::string(entry) + ": unknown exception";
    return status(FABER_STATUS_PANIC);
  }
}

#define FABER_ARG(cond, msg) ::faber::require((cond), FABER_STATUS_INVALID_ARGUMENT, (msg))

}  // namespace faber
