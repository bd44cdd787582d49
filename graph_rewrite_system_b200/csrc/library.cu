// Library-level entry points of libgrs_b200.so.
#include "grs_common.cuh"

extern "C" const char* grs_version(void) {
  return "grs_b200 0.1 sm_100a";
}
