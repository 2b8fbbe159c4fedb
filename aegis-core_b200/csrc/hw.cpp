// Hardware description and device manifest entry points of the C ABI
// (aegis_hw_info_json / aegis_hw_gpu / aegis_hw_cpu / aegis_device_manifest).
// The reference's implementations read Jetson/Tegra sysfs, NVML, thermal
// zones and video engines (src/hw/discover.cpp, src/manifest.cpp); this
// library keeps the same entry points, struct layouts and JSON keys with a
// thin implementation: CUDA device properties, the host CPU count and
// cpufreq limit, and a measured device-to-device copy bandwidth. Fields no
// source here reads are -1 / null.
#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "aegis.h"
#include "capi_error.h"

namespace {

int hw_fail(int status, const char* what) {
  aegis::capi::set_error(what);
  return status;
}

long long read_ll(const char* path) {
  std::ifstream f(path);
  long long v = -1;
  if (f && (f >> v)) return v;
  return -1;
}

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') o += '\\';
    if (static_cast<unsigned char>(c) >= 0x20) o += c;
  }
  return o;
}

int copy_out(const std::string& s, char* buf, size_t buf_len, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (!buf && buf_len == 0) return AEGIS_OK;
  if (!buf) return hw_fail(AEGIS_ERR_INVALID_ARGUMENT, "buf is NULL but buf_len is not 0");
  if (buf_len < s.size() + 1) return hw_fail(AEGIS_ERR_BUFFER_TOO_SMALL, "buffer too small");
  std::memcpy(buf, s.c_str(), s.size() + 1);
  return AEGIS_OK;
}

bool device_ok(int device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return device >= 0 && device < count;
}

aegis_hw_gpu_info gpu_info(int device) {
  aegis_hw_gpu_info r;
  std::memset(&r, 0, sizeof r);
  r.struct_size = uint32_t(sizeof r);
  r.device = device;
  r.max_sm_clock_mhz = -1;
  r.max_mem_clock_mhz = -1;
  r.power_limit_w = -1;
  cudaDeviceProp p{};
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) {
    cudaGetLastError();
    return r;
  }
  r.present = 1;
  r.arch = p.major * 10 + p.minor;
  r.sm_count = p.multiProcessorCount;
  r.regs_per_sm = p.regsPerMultiprocessor;
  r.smem_per_sm = int64_t(p.sharedMemPerMultiprocessor);
  r.smem_per_block = int64_t(p.sharedMemPerBlock);
  r.smem_per_block_optin = int64_t(p.sharedMemPerBlockOptin);
  r.l2_bytes = p.l2CacheSize;
  r.memory_bytes = int64_t(p.totalGlobalMem);
  r.unified = p.integrated;
  r.tma_hardware = r.arch >= 90;
  r.tma_built = 1;
  r.nvml = 0;
  int khz = 0;
  if (cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device) == cudaSuccess && khz > 0) r.max_sm_clock_mhz = khz / 1000;
  if (cudaDeviceGetAttribute(&khz, cudaDevAttrMemoryClockRate, device) == cudaSuccess && khz > 0)
    r.max_mem_clock_mhz = khz / 1000;
  cudaGetLastError();
  std::snprintf(r.name, sizeof r.name, "%.127s", p.name);
  return r;
}

aegis_hw_cpu_info cpu_info() {
  aegis_hw_cpu_info r;
  std::memset(&r, 0, sizeof r);
  r.struct_size = uint32_t(sizeof r);
  const long n = sysconf(_SC_NPROCESSORS_ONLN);
  r.logical_cpus = int32_t(n > 0 ? n : 1);
  r.clusters = 1;
  r.core_types = 1;
  r.performance_cores = r.logical_cpus;
  r.performance_max_khz = read_ll("/sys/devices/system/cpu/cpu0/cpufreq/cpuinfo_max_freq");
  return r;
}

std::string hw_json(int device) {
  const aegis_hw_cpu_info c = cpu_info();
  std::string j = "{\"schema\":\"aegis-hw/1\",\"gpu\":";
  if (device >= 0) {
    const aegis_hw_gpu_info g = gpu_info(device);
    char b[1024];
    std::snprintf(b, sizeof b,
                  "{\"present\":%s,\"device\":%d,\"name\":\"%s\",\"arch\":%d,\"sm_count\":%d,\"regs_per_sm\":%d,"
                  "\"smem_per_sm\":%lld,\"smem_per_block_optin\":%lld,\"l2_bytes\":%lld,\"memory_bytes\":%lld,"
                  "\"unified\":%s,\"tma_hardware\":%s,\"tma_built\":true,\"tcgen05\":%s,\"max_sm_clock_mhz\":%d,"
                  "\"max_mem_clock_mhz\":%d,\"power_limit_w\":null}",
                  g.present ? "true" : "false", g.device, json_escape(g.name).c_str(), g.arch, g.sm_count,
                  g.regs_per_sm, (long long)g.smem_per_sm, (long long)g.smem_per_block_optin, (long long)g.l2_bytes,
                  (long long)g.memory_bytes, g.unified ? "true" : "false", g.tma_hardware ? "true" : "false",
                  g.arch == 100 ? "true" : "false", g.max_sm_clock_mhz, g.max_mem_clock_mhz);
    j += b;
  } else {
    j += "{\"present\":false}";
  }
  char b[512];
  std::snprintf(b, sizeof b,
                ",\"cpu\":{\"logical_cpus\":%d,\"clusters\":[{\"id\":0,\"cpus\":%d}],\"core_types\":[{\"cpus\":%d,"
                "\"max_khz\":%lld,\"performance\":true}],\"isa\":{}},\"memory\":{\"total_bytes\":%lld},"
                "\"thermal\":[],\"video\":{\"nvdec\":null,\"nvenc\":null}}",
                c.logical_cpus, c.logical_cpus, c.logical_cpus, (long long)c.performance_max_khz,
                (long long)sysconf(_SC_PHYS_PAGES) * (long long)sysconf(_SC_PAGE_SIZE));
  j += b;
  return j;
}

struct DeviceGuard {
  int prev = 0;
  bool ok = cudaGetDevice(&prev) == cudaSuccess;
  ~DeviceGuard() {
    if (ok) cudaSetDevice(prev);
  }
};

// Device manifest: properties plus a measured device-to-device copy bandwidth
// (512 MiB, read + write bytes, best of 10 CUDA-event-timed copies).
cudaError_t manifest_json(int device, std::string& out) {
  DeviceGuard guard;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return e;
  cudaDeviceProp p{};
  int rt = 0, drv = 0;
  if ((e = cudaGetDeviceProperties(&p, device)) != cudaSuccess) return e;
  if ((e = cudaRuntimeGetVersion(&rt)) != cudaSuccess) return e;
  if ((e = cudaDriverGetVersion(&drv)) != cudaSuccess) return e;
  const size_t bytes = size_t(512) << 20;
  void *src = nullptr, *dst = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float best = 1e30f;
  auto measure = [&]() -> cudaError_t {
    cudaError_t r;
    if ((r = cudaMalloc(&src, bytes)) != cudaSuccess) return r;
    if ((r = cudaMalloc(&dst, bytes)) != cudaSuccess) return r;
    if ((r = cudaMemset(src, 1, bytes)) != cudaSuccess) return r;
    if ((r = cudaEventCreate(&e0)) != cudaSuccess) return r;
    if ((r = cudaEventCreate(&e1)) != cudaSuccess) return r;
    for (int i = 0; i < 11; ++i) {
      cudaEventRecord(e0);
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice);
      cudaEventRecord(e1);
      if ((r = cudaEventSynchronize(e1)) != cudaSuccess) return r;
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      if (i > 0) best = std::min(best, ms);
    }
    return cudaGetLastError();
  };
  e = measure();
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFree(src);
  cudaFree(dst);
  if (e != cudaSuccess) return e;
  const double gbps = 2.0 * double(bytes) / (double(best) * 1e-3) / 1e9;
  char b[1024];
  std::snprintf(b, sizeof b,
                "{\"schema\":\"aegis-manifest/1\",\"device\":%d,\"name\":\"%s\",\"sm_arch\":%d,\"sm_count\":%d,"
                "\"memory_bytes\":%llu,\"l2_bytes\":%d,\"smem_per_block_optin\":%zu,\"cuda_runtime\":%d,"
                "\"cuda_driver\":%d,\"measured_d2d_bw_gbps\":%.1f}",
                device, json_escape(p.name).c_str(), p.major * 10 + p.minor, p.multiProcessorCount,
                (unsigned long long)p.totalGlobalMem, p.l2CacheSize, p.sharedMemPerBlockOptin, rt, drv, gbps);
  out = b;
  return cudaSuccess;
}

}  // namespace

extern "C" {

int aegis_hw_info_json(int device, char* buf, size_t buf_len, size_t* needed) {
  thread_local bool pending = false;
  thread_local int pending_device = 0;
  thread_local std::string snapshot;
  if (!buf && buf_len != 0) return hw_fail(AEGIS_ERR_INVALID_ARGUMENT, "buf is NULL but buf_len is not 0");
  if (device < -1 || (device >= 0 && !device_ok(device))) return hw_fail(AEGIS_ERR_NO_DEVICE, "no such CUDA device");
  if (!(buf && pending && pending_device == device)) snapshot = hw_json(device);
  pending = buf == nullptr;
  pending_device = device;
  return copy_out(snapshot, buf, buf_len, needed);
}

int aegis_hw_gpu(int device, aegis_hw_gpu_info* out) {
  if (!out || out->struct_size < sizeof(uint32_t)) return hw_fail(AEGIS_ERR_INVALID_ARGUMENT, "out is NULL or struct_size unset");
  if (!device_ok(device)) return hw_fail(AEGIS_ERR_NO_DEVICE, "no such CUDA device");
  const aegis_hw_gpu_info r = gpu_info(device);
  const uint32_t want = out->struct_size;
  const uint32_t n = want < sizeof r ? want : uint32_t(sizeof r);
  std::memcpy(out, &r, n);
  out->struct_size = n;
  return AEGIS_OK;
}

int aegis_hw_cpu(aegis_hw_cpu_info* out) {
  if (!out || out->struct_size < sizeof(uint32_t)) return hw_fail(AEGIS_ERR_INVALID_ARGUMENT, "out is NULL or struct_size unset");
  const aegis_hw_cpu_info r = cpu_info();
  const uint32_t want = out->struct_size;
  const uint32_t n = want < sizeof r ? want : uint32_t(sizeof r);
  std::memcpy(out, &r, n);
  out->struct_size = n;
  return AEGIS_OK;
}

int aegis_device_manifest(int device, char* buf, size_t buf_len, size_t* needed) {
  static std::mutex mu;
  static std::map<int, std::string> cache;
  if (!device_ok(device)) return hw_fail(AEGIS_ERR_NO_DEVICE, "no such CUDA device");
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it == cache.end()) {
    std::string j;
    const cudaError_t e = manifest_json(device, j);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return hw_fail(e == cudaErrorMemoryAllocation ? AEGIS_ERR_OUT_OF_MEMORY : AEGIS_ERR_CUDA, cudaGetErrorString(e));
    }
    it = cache.emplace(device, std::move(j)).first;
  }
  return copy_out(it->second, buf, buf_len, needed);
}

}  // extern "C"
