// No C++ exception may leave the C ABI: every entry point that allocates runs
// its body through guarded(), which turns an exception into a status code and
// a ws_last_error() message.
#pragma once
#include <exception>
#include <new>

#include "../../include/warpshift_b200.h"

namespace ws {

void set_last_error(const char* msg);

template <class F>
inline int guarded(F&& body) noexcept {
  try {
    return body();
  } catch (const std::bad_alloc&) {
    set_last_error("out of host memory");
    return WS_ERR_NOMEM;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return WS_ERR_STATE;
  } catch (...) {
    set_last_error("internal error");
    return WS_ERR_STATE;
  }
}

}  // namespace ws
