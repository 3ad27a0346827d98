// Library identity and status strings of the C ABI.
#include "common.cuh"

extern "C" int gsq_abi_version(void) { return 2; }

extern "C" const char* gsq_status_string(int status) {
  switch (status) {
    case GSQ_OK: return "ok";
    case GSQ_EINVAL: return "invalid argument";
    case GSQ_ECUDA: return "CUDA error";
    case GSQ_ETIMEOUT: return "bounded device wait timed out";
    case GSQ_ENOTSUP: return "not supported by this build";
    default: return "unknown status";
  }
}
