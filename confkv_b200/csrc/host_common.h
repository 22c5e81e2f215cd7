// Host-side pieces shared by the translation units of libgpu_aesgcm.so: the
// key handle, the device guard, launch helpers and the per-device set-up.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "gpu_aesgcm_api.h"
#include "host_crypto.h"
#include "kernels.cuh"

namespace confkv {
namespace host {

constexpr size_t kFrameOverhead = 29;
constexpr uint64_t kMaxBlocks = 0xfffffffeull;
constexpr int kSlots = 1024;  // accumulation slots of a key handle: one per stream it is used on
constexpr int kMaxDevices = 64;

struct KeyHandle {
    int device = 0;
    int num_sms = 0;
    uint32_t rk[confkv::kRoundKeyWords];
    uint8_t* d_mem = nullptr;  // one allocation: tables + slots
    dev::KeyTables kt{};
    confkv::ClmulConst open_cm{};  // the batched GHASH passes' chain multiplier, integer-pipe form
    dev::Slot* slots = nullptr;
    // Stream -> its slot. Calls on one stream never overlap on the device
    // (each kernel touches the slot only after griddepcontrol.wait, i.e.
    // after the previous call's kernels completed), so they share it.
    std::mutex slot_mu;
    std::unordered_map<cudaStream_t, uint32_t> stream_slot;
};

// Makes `target` the current device for the scope of a call and restores
// the caller's device afterwards.
class DeviceGuard {
public:
    explicit DeviceGuard(int target)
    {
        if (cudaGetDevice(&old_) != cudaSuccess) {
            ok_ = false;
            return;
        }
        if (old_ != target) {
            ok_ = cudaSetDevice(target) == cudaSuccess;
            changed_ = ok_;
        }
    }
    ~DeviceGuard()
    {
        if (changed_) {
            cudaSetDevice(old_);
        }
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;
    bool ok() const { return ok_; }

private:
    int old_ = 0;
    bool changed_ = false;
    bool ok_ = true;
};

inline int cuda_rc(cudaError_t e)
{
    return e == cudaSuccess ? LMCACHE_GPU_AESGCM_OK : LMCACHE_GPU_AESGCM_ERR_CUDA;
}

// Bytes between the start of a block's dynamic shared memory and
// dev::kSmemLayoutBase, where every kernel's shared layout begins
// (dev::layout_smem). Set from the probe kernel's reading on the first
// configured device: 1 KiB on sm_100a with this driver, where dynamic shared
// memory starts at window address 0x400.
uint32_t layout_pad();

// Records the window address of dynamic shared memory read by
// smem_base_probe_kernel on a device. False (the device is refused) when it
// lies above dev::kSmemLayoutBase, is not 16-byte aligned, or differs from
// the address another device reported.
bool record_layout_base(unsigned int window_base);

// Shared bytes to request for a kernel whose layout takes `layout_bytes`
// (0 for kernels without a shared layout).
inline uint32_t launch_smem(uint32_t layout_bytes)
{
    return layout_bytes == 0 ? 0u : layout_bytes + layout_pad();
}

// Opts `kernel` into the dynamic shared memory of a layout of `bytes` plus the gap.
template <class K>
cudaError_t allow_smem(K kernel, uint32_t bytes)
{
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(launch_smem(bytes)));
}

// Launch with programmatic stream serialization (see pdl_release/pdl_wait):
// the kernel may start while the previous kernel on the stream drains.
// `smem` is the kernel's layout size; the gap before the layout is added here.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), uint32_t grid, uint32_t block, uint32_t smem, cudaStream_t s,
                       Args&&... args)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = launch_smem(smem);
    cfg.stream = s;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Opts every kernel of the library into its dynamic shared memory and checks
// the shared-memory layout, once per device (gpu_aesgcm.cu).
cudaError_t configure_device(int device);

// The batched kernels' part of configure_device (batch.cu).
cudaError_t configure_batch_kernels();

}  // namespace host
}  // namespace confkv
