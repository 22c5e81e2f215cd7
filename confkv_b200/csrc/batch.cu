// Batched seal / open entry points (extensions of the C-ABI): the kernels
// are in batch.cuh; this translation unit holds their launch, the
// descriptor checks made on the host and the workspace size.
#include <cstddef>
#include <cstdlib>
#include <cstring>

#include "batch.cuh"
#include "gpu_aesgcm_api.h"
#include "host_common.h"

namespace dev = confkv::dev;
using namespace confkv::host;

static_assert(sizeof(lmcache_gpu_aesgcm_batch_item) == sizeof(dev::BatchItem), "descriptor size");
static_assert(offsetof(lmcache_gpu_aesgcm_batch_item, auth_ok) == offsetof(dev::BatchItem, auth_ok),
              "descriptor layout");
static_assert(offsetof(lmcache_gpu_aesgcm_batch_item, iv) == offsetof(dev::BatchItem, iv), "descriptor layout");
static_assert(offsetof(lmcache_gpu_aesgcm_batch_item, status) == offsetof(dev::BatchItem, status),
              "descriptor layout");
static_assert(offsetof(dev::BatchHeader, fault) == LMCACHE_GPU_AESGCM_BATCH_FAULT_OFFSET, "fault word offset");
static_assert(offsetof(dev::BatchHeader, seal_two_pass) == 60, "the GPU tests read the seal design at byte 60");

cudaError_t confkv::host::configure_batch_kernels()
{
    cudaError_t e = allow_smem(dev::seal_batch_kernel, dev::kSealBatchSmem);
    if (e == cudaSuccess) {
        e = allow_smem(dev::seal_ghash_batch_kernel, dev::kOpenBatchSmem);
    }
    if (e == cudaSuccess) {
        e = allow_smem(dev::open_ghash_batch_kernel, dev::kOpenBatchSmem);
    }
    if (e == cudaSuccess) {
        e = allow_smem(dev::open_ctr_batch_kernel, dev::kCtrBatchSmem);
    }
    return e;
}

namespace {

// Test-only: CONFKV_B200_TEST_HANDOFF_STALL=1 makes the batched seal's power
// warps stop taking hand-offs and shortens the hand-off waits to
// kInjectedWaitNs, so the row warps' waits run out and the call reports a
// fault in the workspace instead of hanging (tests/test_gpu_batch.py).
constexpr unsigned long long kInjectedWaitNs = 50ull * 1000ull * 1000ull;

bool handoff_stall_injected()
{
    const char* v = std::getenv("CONFKV_B200_TEST_HANDOFF_STALL");
    return v != nullptr && v[0] == '1';
}

// Host checks, then: plan (one CTA) -> seal_batch_kernel, or plan ->
// open_ghash_batch_kernel -> open_ctr_batch_kernel, all with programmatic
// stream serialization so each kernel's table fill overlaps its predecessor.
int batch_launch(lmcache_gpu_aesgcm_key_t key, lmcache_gpu_aesgcm_batch_item* items, size_t count,
                 void* workspace, size_t workspace_bytes, void* stream_ptr, bool open)
{
    if (key == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    if (count == 0) {
        return LMCACHE_GPU_AESGCM_OK;
    }
    if (items == nullptr || workspace == nullptr || count > dev::kBatchMaxItems ||
        (reinterpret_cast<uintptr_t>(items) & 15u) != 0 || (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0 ||
        workspace_bytes < dev::batch_workspace_bytes(count)) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    auto* h = reinterpret_cast<KeyHandle*>(key);
    DeviceGuard guard(h->device);
    if (!guard.ok()) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_ptr);
    auto* d_items = reinterpret_cast<dev::BatchItem*>(items);
    auto* ws = static_cast<uint8_t*>(workspace);
    const int sms = h->num_sms < dev::kBatchMaxSms ? h->num_sms : dev::kBatchMaxSms;
    if (launch_pdl(dev::batch_plan_kernel, 1, dev::kPlanThreads, 0, s, d_items, static_cast<uint32_t>(count), ws,
                   open ? 1 : 0, static_cast<uint32_t>(sms)) != cudaSuccess) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    dev::BatchArgs ba{};
    ba.items = d_items;
    ba.ws = ws;
    ba.count = static_cast<uint32_t>(count);
    ba.stall = handoff_stall_injected() ? 1u : 0u;
    ba.wait_ns = ba.stall != 0u ? kInjectedWaitNs : dev::kWaitLimitNs;
    std::memcpy(ba.rk, h->rk, sizeof(ba.rk));
    ba.kt = h->kt;
    ba.open_cm = h->open_cm;
    const uint32_t grid = static_cast<uint32_t>(h->num_sms);
    int rc;
    if (!open) {
        // the plan picks fused or two passes; seal_ghash_batch_kernel returns
        // at once after a fused seal
        if (launch_pdl(dev::seal_batch_kernel, grid, dev::kSealThreads, dev::kSealBatchSmem, s, ba) != cudaSuccess) {
            rc = LMCACHE_GPU_AESGCM_ERR_CUDA;
        } else {
            rc = cuda_rc(launch_pdl(dev::seal_ghash_batch_kernel, grid, dev::kSealThreads, dev::kOpenBatchSmem, s, ba));
        }
    } else if (launch_pdl(dev::open_ghash_batch_kernel, grid, dev::kSealThreads, dev::kOpenBatchSmem, s, ba) !=
               cudaSuccess) {
        rc = LMCACHE_GPU_AESGCM_ERR_CUDA;
    } else {
        rc = cuda_rc(launch_pdl(dev::open_ctr_batch_kernel, grid, dev::kCtrThreads, dev::kCtrBatchSmem, s, ba));
    }
    std::memset(ba.rk, 0, sizeof(ba.rk));
    return rc;
}

}  // namespace

extern "C" size_t lmcache_gpu_aes128gcm_batch_workspace_size(size_t count)
{
    return count > dev::kBatchMaxItems ? 0 : dev::batch_workspace_bytes(count);
}

extern "C" int lmcache_gpu_aes128gcm_seal_batch_async(lmcache_gpu_aesgcm_key_t key,
                                                      lmcache_gpu_aesgcm_batch_item* items, size_t count,
                                                      void* workspace, size_t workspace_bytes, void* stream)
{
    return batch_launch(key, items, count, workspace, workspace_bytes, stream, false);
}

extern "C" int lmcache_gpu_aes128gcm_open_batch_async(lmcache_gpu_aesgcm_key_t key,
                                                      lmcache_gpu_aesgcm_batch_item* items, size_t count,
                                                      void* workspace, size_t workspace_bytes, void* stream)
{
    return batch_launch(key, items, count, workspace, workspace_bytes, stream, true);
}
