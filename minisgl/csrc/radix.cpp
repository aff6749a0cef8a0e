// Host-side helpers for the radix prefix cache.
//
// fast_compare_key is the native key comparison the reference exposes from
// python/minisgl/kernel/csrc/src/radix.cpp:12-44 (first mismatching position
// of two 1-D CPU integer tensors). Here it is plain C++ over raw pointers,
// called through the pybind layer in binding.cpp.
#include <algorithm>
#include <cstdint>

namespace minisgl {

template <typename A, typename B>
static int64_t mismatch_impl(const A* a, int64_t na, const B* b, int64_t nb) {
  const int64_t n = std::min(na, nb);
  int64_t i = 0;
  // 8-way unrolled scan; the common case is a long equal run
  for (; i + 8 <= n; i += 8) {
    if (a[i] != b[i] || a[i + 1] != b[i + 1] || a[i + 2] != b[i + 2] || a[i + 3] != b[i + 3] ||
        a[i + 4] != b[i + 4] || a[i + 5] != b[i + 5] || a[i + 6] != b[i + 6] ||
        a[i + 7] != b[i + 7])
      break;
  }
  for (; i < n; ++i)
    if (a[i] != b[i]) return i;
  return n;
}

// elem sizes: 4 (int32) or 8 (int64)
int64_t compare_key_raw(const void* a, int64_t na, int ea, const void* b, int64_t nb, int eb) {
  if (ea == 4 && eb == 4)
    return mismatch_impl(static_cast<const int32_t*>(a), na, static_cast<const int32_t*>(b), nb);
  if (ea == 8 && eb == 8)
    return mismatch_impl(static_cast<const int64_t*>(a), na, static_cast<const int64_t*>(b), nb);
  if (ea == 4 && eb == 8)
    return mismatch_impl(static_cast<const int32_t*>(a), na, static_cast<const int64_t*>(b), nb);
  return mismatch_impl(static_cast<const int64_t*>(a), na, static_cast<const int32_t*>(b), nb);
}

}  // namespace minisgl
