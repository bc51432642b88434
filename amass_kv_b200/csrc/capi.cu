// Library-level C ABI: status strings, version, one-time device setup.
#include "common.cuh"

extern "C" const char* amass_status_string(int status) {
  switch (status) {
    case AMASS_OK: return "ok";
    case AMASS_ERR_ARG: return "invalid argument (null pointer, size or stride)";
    case AMASS_ERR_UNSUPPORTED: return "geometry outside the compiled variants";
    case AMASS_ERR_CAPACITY: return "caller buffer too small";
    case AMASS_ERR_CUDA: return "CUDA launch error";
  }
  return "unknown status";
}

extern "C" int amass_version(void) { return 1; }

extern "C" int amass_init(void) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return AMASS_ERR_CUDA;
  (void)amass::num_sms();
  return AMASS_OK;
}
