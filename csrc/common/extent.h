// Host helper for the bounds-checked build: how many elements a kernel may
// touch through a tensor's data pointer.
#pragma once

#include <torch/extension.h>

namespace h3 {

// Elements from `t`'s first element to the end of its storage (the real
// allocation, not the view's logical size).
inline long extent_of(const at::Tensor& t) {
  const long bytes = static_cast<long>(t.storage().nbytes()) -
                     static_cast<long>(t.storage_offset()) * static_cast<long>(t.element_size());
  return bytes / static_cast<long>(t.element_size());
}

}  // namespace h3
