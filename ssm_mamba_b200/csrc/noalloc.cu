// Backward selective scan that allocates nothing.
//
// Who needs it: a caller that cannot call cudaMalloc at the point where it runs the
// backward -- a framework or runtime whose own allocator owns every byte of device memory
// (a second allocator would fragment or overrun its pool), or a host language binding that
// reaches this library through a plain C FFI and has no device-allocation API at all.
// ssm_scan_bwd needs a workspace from its caller; this variant instead uses a fixed
// scratch buffer compiled into the library as a file-scope __device__ array, so the
// caller passes only its inputs and outputs.
//
// The array is kStaticScratchBytes (16 MiB) on every GPU that loads the library, held until
// the process exits.  Its last 256 bytes hold the error word of this variant's kernels
// (zero at load; a bounded wait that runs out writes its code there, and
// ssm_check_device_error reads and clears it); the rest is the backward's workspace, so
// shapes whose workspace (ssm_scan_bwd_workspace_size) exceeds kStaticWorkspaceBytes are
// rejected.  The workspace is fully overwritten by every call (the per-tile and per-batch
// partials cover every output element), so nothing in it needs clearing between calls.
// All calls on a device share the array: two calls whose kernels overlap on the GPU
// (different streams, or different host threads) race on it and must be serialised by
// the caller.
//
// The device address of the array is obtained once per device, on that device's first
// call, with cudaGetSymbolAddress (host code cannot use the array's name as a device
// address); the first call on a device should therefore come before any stream capture.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/ssm_b200.h"

namespace ssm {
size_t scan_bwd_workspace_bytes(const ssm_scan_bwd_args* a, int sms);
int scan_bwd_run(const ssm_scan_bwd_args* a, void* workspace, size_t ws_bytes, int* err_word, int sms,
                 void* stream);
void set_last_error(const char* msg);
}  // namespace ssm

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;
constexpr size_t kStaticWorkspaceBytes = kStaticScratchBytes - 256;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct StaticDev {
    bool ready = false;
    unsigned char* base = nullptr;
    int sms = 0;
};
std::mutex g_static_mu;
StaticDev g_static_dev[64];

int static_setup(StaticDev** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        ssm::set_last_error("ssm_scan_bwd_noalloc: no current CUDA device");
        return SSM_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lk(g_static_mu);
    StaticDev& s = g_static_dev[dev];
    if (!s.ready) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || p == nullptr) {
            ssm::set_last_error("ssm_scan_bwd_noalloc: cudaGetSymbolAddress of the static scratch failed");
            return SSM_ERR_CUDA;
        }
        if (cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            ssm::set_last_error("ssm_scan_bwd_noalloc: cudaDeviceGetAttribute failed");
            return SSM_ERR_CUDA;
        }
        s.base = static_cast<unsigned char*>(p);
        s.ready = true;
    }
    *out = &s;
    return SSM_OK;
}

}  // namespace

namespace ssm {

// Device address of the current device's noalloc error word, or nullptr when no
// ssm_scan_bwd_noalloc call has set that device up (its kernels cannot have written it).
int* noalloc_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_static_mu);
    const StaticDev& s = g_static_dev[dev];
    return s.ready ? reinterpret_cast<int*>(s.base + kStaticWorkspaceBytes) : nullptr;
}

}  // namespace ssm

extern "C" int ssm_scan_bwd_noalloc(const ssm_scan_bwd_args* args, void* stream) {
    if (!args) {
        ssm::set_last_error("ssm_scan_bwd_noalloc: args is NULL");
        return SSM_ERR_INVALID;
    }
    StaticDev* s = nullptr;
    int rc = static_setup(&s);
    if (rc) return rc;
    const size_t need = ssm::scan_bwd_workspace_bytes(args, s->sms);
    if (need == 0) return ssm::scan_bwd_run(args, nullptr, 0, nullptr, s->sms, stream);  // reports the shape error
    if (need > kStaticWorkspaceBytes) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "ssm_scan_bwd_noalloc: this shape needs %zu bytes of workspace, more than the %zu-byte "
                 "static scratch; use ssm_scan_bwd with a caller-provided workspace",
                 need, kStaticWorkspaceBytes);
        ssm::set_last_error(msg);
        return SSM_ERR_WORKSPACE;
    }
    int* err_word = reinterpret_cast<int*>(s->base + kStaticWorkspaceBytes);
    return ssm::scan_bwd_run(args, s->base, kStaticWorkspaceBytes, err_word, s->sms, stream);
}
