/**
 * @file device.hpp
 * @brief Device discovery and selection (the reference's core/device.hpp
 *        interface: DeviceInfo, DeviceManager and the device:: free functions).
 *
 * Differences from the reference, all B200-driven: sm_100 is recognised
 * (the reference maps every unknown capability, 10.0 included, to SM_70,
 * core/device.hpp:254-263), devices below sm_100 are not "supported" because
 * this build's kernels are sm_100a-only, and DeviceInfo carries what the
 * kernel dispatcher needs (SM count, opt-in shared memory, cluster launch).
 * Properties come from the library (choreo_device_props_get).
 */
#ifndef CHOREO_IR_CORE_DEVICE_HPP
#define CHOREO_IR_CORE_DEVICE_HPP

#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../choreo_b200.h"
#include "config.hpp"
#include "types.hpp"

namespace choreo_ir {
namespace device {

struct DeviceInfo {
  int device_id = -1;
  std::string name;
  ComputeCapability compute_capability = ComputeCapability::SM_70;
  size_t total_memory = 0;
  size_t free_memory = 0;
  int multiprocessor_count = 0;
  int max_threads_per_block = 0;
  int max_shared_memory_per_block = 0;   // opt-in maximum
  int warp_size = 32;
  bool tensor_core_support = false;      // tcgen05 (sm_100)
  bool cluster_launch = false;
};

inline ComputeCapability capability_from(int major, int minor) {
  switch (major * 10 + minor) {
    case 70: return ComputeCapability::SM_70;
    case 75: return ComputeCapability::SM_75;
    case 80: return ComputeCapability::SM_80;
    case 86: return ComputeCapability::SM_86;
    case 89: return ComputeCapability::SM_89;
    case 90: return ComputeCapability::SM_90;
    case 100: return ComputeCapability::SM_100;
    default: return major >= 10 ? ComputeCapability::SM_100 : ComputeCapability::SM_70;
  }
}

class DeviceManager {
 public:
  static DeviceManager& instance() {
    static DeviceManager m;
    return m;
  }

  /// Enumerates sm_100 devices and makes the first one current.
  bool initialize() {
    std::lock_guard<std::mutex> lk(mu_);
    if (initialized_) return true;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
      cudaGetLastError();
      return false;
    }
    infos_.clear();
    for (int i = 0; i < count; ++i) {
      DeviceInfo info;
      if (!query(i, info)) continue;
      if (info.compute_capability != ComputeCapability::SM_100) continue;
      infos_.push_back(info);
    }
    if (infos_.empty()) return false;
    current_ = infos_.front().device_id;
    cudaSetDevice(current_);
    initialized_ = true;
    return true;
  }

  /// Forgets the device list. Unlike the reference (core/device.hpp:102-107)
  /// this does not cudaDeviceReset(): other owners of the context (a
  /// framework, another library) would lose their allocations.
  void finalize() {
    std::lock_guard<std::mutex> lk(mu_);
    initialized_ = false;
    infos_.clear();
  }

  int get_device_count() const { return static_cast<int>(infos_.size()); }

  const DeviceInfo& get_device_info(int device_id) const {
    for (const auto& i : infos_)
      if (i.device_id == device_id) return i;
    throw std::runtime_error("Device not found: " + std::to_string(device_id));
  }

  bool set_device(int device_id) {
    if (!initialized_) return false;
    for (const auto& i : infos_) {
      if (i.device_id == device_id) {
        if (cudaSetDevice(device_id) != cudaSuccess) return false;
        current_ = device_id;
        return true;
      }
    }
    return false;
  }

  int get_current_device() const { return current_; }

  bool is_tensor_core_supported() const {
    if (!initialized_) return false;
    try {
      return get_device_info(current_).tensor_core_support;
    } catch (const std::exception&) {
      return false;
    }
  }

  ComputeCapability get_compute_capability() const {
    if (!initialized_) return ComputeCapability::SM_70;
    try {
      return get_device_info(current_).compute_capability;
    } catch (const std::exception&) {
      return ComputeCapability::SM_70;
    }
  }

  void synchronize() {
    if (initialized_) cudaDeviceSynchronize();
  }

  bool is_initialized() const { return initialized_; }

 private:
  DeviceManager() = default;

  static bool query(int id, DeviceInfo& info) {
    choreo_device_props p;
    if (choreo_device_props_get(id, &p) != CHOREO_OK) return false;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, id) != cudaSuccess) return false;
    info.device_id = id;
    info.name = p.name;
    info.compute_capability = capability_from(p.cc_major, p.cc_minor);
    info.total_memory = static_cast<size_t>(p.total_mem);
    info.multiprocessor_count = p.sm_count;
    info.max_threads_per_block = prop.maxThreadsPerBlock;
    info.max_shared_memory_per_block = p.max_smem_optin;
    info.warp_size = prop.warpSize;
    info.tensor_core_support = p.cc_major >= 10;
    info.cluster_launch = p.cluster_launch != 0;
    int prev = 0;
    cudaGetDevice(&prev);
    size_t free_b = 0, total_b = 0;
    if (cudaSetDevice(id) == cudaSuccess && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess)
      info.free_memory = free_b;
    cudaSetDevice(prev);
    return true;
  }

  std::mutex mu_;
  bool initialized_ = false;
  int current_ = 0;
  std::vector<DeviceInfo> infos_;
};

inline bool initialize() { return DeviceManager::instance().initialize(); }
inline void finalize() { DeviceManager::instance().finalize(); }
inline int get_current_device() { return DeviceManager::instance().get_current_device(); }
inline bool set_device(int device_id) { return DeviceManager::instance().set_device(device_id); }
inline void synchronize() { DeviceManager::instance().synchronize(); }
inline bool is_tensor_core_supported() { return DeviceManager::instance().is_tensor_core_supported(); }
inline bool supports_tensor_core() { return is_tensor_core_supported(); }
inline ComputeCapability get_compute_capability() { return DeviceManager::instance().get_compute_capability(); }
inline int get_device_count() { return DeviceManager::instance().get_device_count(); }
inline const DeviceInfo& get_device_info(int device_id = -1) {
  if (device_id == -1) device_id = get_current_device();
  return DeviceManager::instance().get_device_info(device_id);
}

}  // namespace device
}  // namespace choreo_ir

#endif  // CHOREO_IR_CORE_DEVICE_HPP
