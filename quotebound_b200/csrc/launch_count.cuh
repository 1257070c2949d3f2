// Process-wide count of the kernels this library has launched (read with qb_gdn_launches()).
#pragma once
#include <stdint.h>

namespace qbgdn {
void note_launch(int64_t n = 1);
int64_t launches();
}  // namespace qbgdn
