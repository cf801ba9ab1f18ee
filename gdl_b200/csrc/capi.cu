// capi.cu -- library-level C entry points (version, status names, device check).
#include "common.cuh"

extern "C" int gdl_version(void) { return 100; }  // 0.1.0

extern "C" const char *gdl_status_string(int status) {
    switch (status) {
    case GDL_OK: return "ok";
    case GDL_ERR_INVALID: return "invalid argument";
    case GDL_ERR_WORKSPACE: return "workspace too small";
    case GDL_ERR_CUDA: return "CUDA error";
    case GDL_ERR_UNSUPPORTED: return "unsupported device or configuration";
    case GDL_ERR_OVERFLOW: return "size exceeds the kernel's index range";
    case GDL_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
    }
}

extern "C" int gdl_check_device(int device) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return GDL_ERR_CUDA;
    if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return GDL_ERR_CUDA;
    return (major == 10 && minor == 0) ? GDL_OK : GDL_ERR_UNSUPPORTED;
}
