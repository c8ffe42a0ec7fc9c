// Host-side parsing of the tensor-parallel exchange arguments (see Xchg in
// common.cuh).  Python passes them as a list of int64:
//   [wait_flag_ptr, wait_delta, sig_flag_ptr, sig_counter_ptr, sig_delta, sdev_ptr, peer_out_ptr]
// An empty list means "no exchange".
#pragma once
#include <torch/extension.h>

#include <cstdint>
#include <vector>

#include "common.cuh"

namespace sb {

inline Xchg xchg_from(const std::vector<int64_t>& v) {
  Xchg x{};
  if (v.empty()) return x;
  TORCH_CHECK(v.size() >= 7, "exchange args: [wait_flag, wait_delta, sig_flag, sig_counter, sig_delta, sdev, peer_out]");
  x.wait_flag = reinterpret_cast<const int*>(v[0]);
  x.wait_delta = static_cast<int>(v[1]);
  x.sig_flag = reinterpret_cast<int*>(v[2]);
  x.sig_counter = reinterpret_cast<int*>(v[3]);
  x.sig_delta = static_cast<int>(v[4]);
  x.sdev = reinterpret_cast<const int*>(v[5]);
  x.peer_out = reinterpret_cast<void*>(v[6]);
  TORCH_CHECK((x.wait_flag == nullptr && x.sig_flag == nullptr) || x.sdev != nullptr,
              "exchange: a wait or signal needs the device step block");
  TORCH_CHECK(x.sig_flag == nullptr || x.sig_counter != nullptr, "exchange: a signal needs a CTA counter");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.peer_out) % 16 == 0, "exchange: peer destination must be 16-byte aligned");
  return x;
}

}  // namespace sb
