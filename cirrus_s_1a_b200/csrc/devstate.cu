// Per-device launch state of the library.
//
// Kernel attributes (the dynamic shared-memory opt-in) and occupancy are
// properties of a kernel on one device, so they are recorded per (kernel,
// device) under one mutex: a process may drive several GPUs from several
// threads, and each device gets its own opt-in the first time a kernel is
// launched there.  The SM count is likewise looked up per device.
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace cb {
namespace {

std::mutex g_mu;
std::map<std::pair<const void*, int>, int> g_smem;      // (kernel, device) -> bytes opted in
std::map<std::pair<const void*, int>, int> g_resident;  // (kernel, device) -> CTAs per SM
std::map<int, int> g_sms;                              // device -> SM count
std::map<std::pair<const void*, int>, int> g_clusters;  // (kernel, device) -> resident clusters
std::map<int, bool> g_coop_refused;                    // device -> cooperative cluster launch refused

int current_device() {
  int dev = -1;
  return cudaGetDevice(&dev) == cudaSuccess ? dev : -1;
}

}  // namespace

int ensure_smem_attr(const void* fn, int bytes) {
  const int dev = current_device();
  if (dev < 0) return CB_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_smem.find({fn, dev});
  if (it != g_smem.end() && it->second >= bytes) return CB_OK;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return CB_ERR_CUDA;
  g_smem[{fn, dev}] = bytes;
  return CB_OK;
}

int resident_ctas(const void* fn, int threads, int smem_bytes) {
  const int dev = current_device();
  if (dev < 0) return 0;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_resident.find({fn, dev});
  if (it != g_resident.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem_bytes) != cudaSuccess) per_sm = 0;
  g_resident[{fn, dev}] = per_sm;
  return per_sm;
}

int resident_clusters(const void* fn, int threads, int smem_bytes, int cluster) {
  const int dev = current_device();
  if (dev < 0) return 0;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_clusters.find({fn, dev});
  if (it != g_clusters.end()) return it->second;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(cluster);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  g_clusters[{fn, dev}] = n;
  return n;
}

bool cooperative_clusters_ok() {
  // CIRRUS_B200_PLAIN_CLUSTERS=1 launches the persistent kernel without the
  // cooperative attribute (profilers that cannot replay cooperative cluster
  // launches); the grid is sized by the occupancy query either way
  static const bool plain = [] {
    const char* e = std::getenv("CIRRUS_B200_PLAIN_CLUSTERS");
    return e != nullptr && e[0] == '1';
  }();
  if (plain) return false;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_coop_refused.find(dev);
  return it == g_coop_refused.end() || !it->second;
}

void note_cooperative_clusters_refused() {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_mu);
  g_coop_refused[dev] = true;
}

int num_sms() {
  const int dev = current_device();
  if (dev < 0) return 148;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_sms.find(dev);
  if (it != g_sms.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  g_sms[dev] = n;
  return n;
}

}  // namespace cb
