// Per-device status word shared by every kernel of the library.  A kernel
// whose bounded wait runs out (or whose checked index is out of range)
// writes a DSV3_ERR_* code here instead of hanging or trapping; the host
// reads it with `status_read()` after a step and raises.
#pragma once
#include <cstdint>

namespace dsv3 {
unsigned int* status_ptr();          // device pointer for the current device
unsigned int status_read();          // synchronous read (syncs the current stream)
void status_reset();                 // zero the word (stream-ordered)
}  // namespace dsv3
