// htrc_flat_forward_static_ws: the forward pass with its workspace in a file-scope device array.
//
// For callers that cannot allocate device memory: code that runs where cudaMalloc is not available
// or not allowed (for example a plugin host that owns every device allocation and hands the plugin
// only its input and output buffers, or an embedding that must not grow the device footprint after
// start-up).  Such a caller still passes q, k, v (and the optional tail) and the out / lse buffers;
// the scratch the operator needs between its kernels (the INT8 keys, tile codes and the per-(tile,
// leaf) state) lives in kStaticWorkspaceBytes of device memory declared in this file.  Every GPU that
// loads this part of the library holds that array until the process exits.
//
// The array is shared by every call on a device and keeps the last call's contents; calls that
// overlap on the GPU (different streams, or different host threads) race on it, so issue them in
// order on one stream.  The device status word at the start of the array is cleared by each call;
// htrc_flat_static_ws_status reads it (and clears it) after a call.
// The first call on each device looks up the array's device address (cudaGetSymbolAddress, with that
// device current); make that first call before any stream capture.  The address is cached for the life
// of the process, so this entry point must not be used across cudaDeviceReset (which reloads the module
// elsewhere).  No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kStaticWorkspaceBytes = size_t(64) << 20;   // 64 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_static_workspace[kStaticWorkspaceBytes];

void* g_addr[kMaxDevices] = {};
std::mutex g_mutex;

// device address of the static workspace on the current device (looked up once per device)
int static_workspace(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return HTRC_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_workspace) != cudaSuccess || p == nullptr) return HTRC_ERR_CUDA;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return HTRC_OK;
}

}  // namespace

extern "C" {

int htrc_flat_forward_static_ws(const HtrcFlatArgs* args, htrc_stream_t stream) {
  if (args == nullptr) return HTRC_ERR_ARG;
  size_t need = 0;
  int rc = htrc_flat_workspace_size(args, &need);
  if (rc != HTRC_OK) return rc;
  if (need > kStaticWorkspaceBytes) return HTRC_ERR_TOO_LARGE;
  void* ws = nullptr;
  if ((rc = static_workspace(&ws)) != HTRC_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the status word (first 4 bytes of the workspace layout) must start at zero
  if (cudaMemsetAsync(ws, 0, 256, st) != cudaSuccess) return HTRC_ERR_CUDA;
  HtrcFlatArgs a = *args;
  a.workspace = ws;
  a.workspace_bytes = kStaticWorkspaceBytes;
  return htrc_flat_forward(&a, stream);
}

int htrc_flat_static_ws_status(int32_t* status_out, htrc_stream_t stream) {
  if (status_out == nullptr) return HTRC_ERR_ARG;
  void* ws = nullptr;
  int rc = static_workspace(&ws);
  if (rc != HTRC_OK) return rc;
  // same read-and-clear as htrc_flat_status, on the status word at the start of the static array
  return htrc_flat_status(ws, status_out, stream);
}

}  // extern "C"
