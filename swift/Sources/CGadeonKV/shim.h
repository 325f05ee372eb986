/* The C ABI of libgadeonkv.so for SwiftPM's system-library target. */
#include "../../../include/gadeon_kv.h"
