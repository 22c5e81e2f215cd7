/*
 * B200 (sm_100a) AES-128-GCM seal/open engine for persistent KV-cache objects.
 *
 * Drop-in C-ABI for ConfKV's GPU seal path. Every declaration below keeps the
 * name, argument list, return convention and memory-space contract of the
 * reference header experiments/gpu_kv_seal/gpu/gpu_aesgcm_api.h; the line cited
 * beside each is the declaration it replaces.
 *
 * Frame written by seal and consumed by open (reference gpu_aesgcm.cu:14-20):
 *
 *     [version = 1][12-byte IV][ciphertext, P bytes][16-byte GCM tag]
 *
 * AAD is empty, IVs are 96-bit (J0 = IV || 0^31 || 1).
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque key handle (reference gpu_aesgcm_api.h:10). */
typedef void* lmcache_gpu_aesgcm_key_t;

/* Return codes (reference gpu_aesgcm_api.h:12-18). Authentication failure is
 * NOT a return code: open reports it through *auth_ok and a zeroed dst. */
enum {
    LMCACHE_GPU_AESGCM_OK = 0,
    LMCACHE_GPU_AESGCM_ERR_ARGUMENT = -1,
    LMCACHE_GPU_AESGCM_ERR_ALLOC = -2,
    LMCACHE_GPU_AESGCM_ERR_CUDA = -3,
    LMCACHE_GPU_AESGCM_ERR_INTERNAL = -4,
};

/* P + 29 (reference gpu_aesgcm_api.h:20-22). Needs no GPU. */
size_t lmcache_gpu_aesgcm_frame_size(size_t plaintext_len);

/*
 * Expand a 16-byte AES key for `device` (reference gpu_aesgcm_api.h:24-29).
 * Computes H = E_K(0^128) and the GHASH multiplication tables on the host,
 * uploads them once, and synchronises the device before returning.
 * key_len != 16, a null key or a null out -> ERR_ARGUMENT.
 */
int lmcache_gpu_aes128gcm_key_create(const uint8_t* key, size_t key_len, int device,
                                     lmcache_gpu_aesgcm_key_t* out);

/* Free the handle's device memory; a null handle is OK
 * (reference gpu_aesgcm_api.h:31-33). */
int lmcache_gpu_aes128gcm_key_destroy(lmcache_gpu_aesgcm_key_t key);

/*
 * Pre-size per-call workspace for objects up to max_plaintext_len bytes
 * (reference gpu_aesgcm_api.h:35-44). The workspace here is a fixed set of
 * per-handle accumulation slots (1024, one per stream) that key_create
 * already allocates, so this only validates the handle;
 * seal/open never call cudaMalloc.
 */
int lmcache_gpu_aes128gcm_reserve(lmcache_gpu_aesgcm_key_t key, size_t max_plaintext_len);

/*
 * Enqueue seal of P = plaintext_len bytes on `stream` (reference
 * gpu_aesgcm_api.h:46-66). src and dst are DEVICE pointers of any alignment;
 * iv is a HOST pointer to exactly 12 bytes, copied before return; stream is a
 * cudaStream_t cast to void* (null = legacy default stream).
 * dst_capacity < P + 29 or more than 2^32 - 2 blocks -> ERR_ARGUMENT.
 * rc reports only enqueue errors; the caller synchronises.
 *
 * Concurrency (lifts the reference's one-stream-per-handle rule): several
 * streams and host threads may use one handle at once, with any number of
 * calls outstanding. Each stream a handle is used on gets one of the handle's
 * 1024 accumulation slots at its first seal_async / open_async; the calls of
 * one stream share it (they are ordered on the device). A call on a 1025th
 * distinct stream returns ERR_ALLOC. A stream destroyed with calls still
 * pending should not be replaced by a new stream on the same handle before
 * those calls complete (the new stream may get the old one's handle value,
 * and with it its slot).
 */
int lmcache_gpu_aes128gcm_seal_async(lmcache_gpu_aesgcm_key_t key, const void* src,
                                     size_t plaintext_len, void* dst, size_t dst_capacity,
                                     const uint8_t* iv, void* stream);

/*
 * Enqueue authentication-gated open (reference gpu_aesgcm_api.h:68-88).
 * src (frame), dst (plaintext) and auth_ok are DEVICE pointers. frame_len may
 * exceed P + 29 (padded frames); the tag is read at offset 13 + P.
 * *auth_ok becomes 1 when the tag and version byte match, else 0 and the P
 * bytes of dst are zero-filled. Plaintext is written only after the tag has
 * been verified on the device, in stream order.
 */
int lmcache_gpu_aes128gcm_open_async(lmcache_gpu_aesgcm_key_t key, const void* src,
                                     size_t frame_len, void* dst, size_t plaintext_len,
                                     int* auth_ok, void* stream);

/*
 * Seal that allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc when they seal (a server whose
 * memory pool already owns the device's memory, or a thread that must not
 * take cudaMalloc's implicit device synchronisation). It takes the raw
 * 16-byte key instead of a handle, runs on `device`, and writes the same
 * frame as lmcache_gpu_aes128gcm_seal_async. Its only working memory is one
 * file-scope __device__ array of 234,752 bytes that every GPU loading this
 * library holds until the process exits; it calls no cudaMalloc or cudaFree.
 *
 * - plaintext_len above 1 GiB (2^30 bytes) -> ERR_ARGUMENT (the array holds
 *   GHASH tables for objects up to that size); other argument rules as seal.
 * - The first call on a device sets up that device (resolves the array's
 *   address, opts the kernels into their shared memory, copies in the AES
 *   tables, checks the layout) and waits for it; make that first call before
 *   any stream capture.
 * - All calls share the array. Each call enqueues a small kernel ahead of
 *   the seal that compares the key's H = E_K(0^128) with the one the array's
 *   GHASH tables were built for and rebuilds them on a mismatch, and clears
 *   the accumulation slot, all in stream order. The host keeps no key
 *   material between calls; the array keeps the last key's GHASH tables (and
 *   that H) until another key replaces them or the process exits.
 * - Calls from several host threads on one stream are safe (each call's two
 *   launches stay adjacent). Calls whose work overlaps on the GPU (other
 *   streams, unordered) race on the array; issue them on one stream or wait
 *   for the previous call.
 */
int lmcache_gpu_aes128gcm_seal_noalloc(const uint8_t* key, size_t key_len, const void* src,
                                       size_t plaintext_len, void* dst, size_t dst_capacity,
                                       const uint8_t* iv, int device, void* stream);

/*
 * Batched seal / open. Extensions: no counterpart in the reference, whose
 * callers enqueue one seal_async / open_async per object.
 *
 * One call covers `count` objects of any sizes (0 included) and alignments
 * with a fixed number of launches (3 each), so thousands of small
 * objects cost one pass over the GPU instead of one launch sequence each.
 * Frames, tags and open's gating are exactly those of seal_async/open_async.
 *
 * items: DEVICE array of `count` descriptors, 16-byte aligned. The device
 *   checks each descriptor by the rules of seal_async / open_async and writes
 *   its `status`: 0, or ERR_ARGUMENT, in which case that object is skipped:
 *   nothing of it is written, except that a rejected open descriptor with a
 *   non-null auth_ok gets *auth_ok = 0 (so a reused verdict buffer never
 *   keeps an earlier call's 1 next to an unwritten dst).
 * workspace: DEVICE buffer, 16-byte aligned, at least
 *   lmcache_gpu_aes128gcm_batch_workspace_size(count) bytes, any contents; the
 *   call owns it until its work on `stream` completes (one call at a time).
 *   After the call, the uint32 at byte offset
 *   LMCACHE_GPU_AESGCM_BATCH_FAULT_OFFSET is nonzero if a work kernel gave up
 *   on one of its internal waits (bounded; a fault, never expected): the
 *   call's frames, tags and verdicts are then invalid.
 * Host-side errors (null key/items/workspace, misalignment, a short
 * workspace, count above 2^20) return ERR_ARGUMENT before any launch;
 * count == 0 is a no-op.
 */
typedef struct lmcache_gpu_aesgcm_batch_item {
    const void* src;          /* seal: plaintext; open: frame (DEVICE) */
    void* dst;                /* seal: frame; open: plaintext (DEVICE) */
    uint64_t plaintext_len;   /* P */
    uint64_t capacity;        /* seal: dst capacity; open: frame length */
    int* auth_ok;             /* open: DEVICE int, 1 = authentic, else 0; seal: unused */
    uint8_t iv[12];           /* seal: the object's IV; open: unused (read from the frame) */
    int32_t status;           /* written by the device */
    uint64_t reserved;        /* set to 0 */
} lmcache_gpu_aesgcm_batch_item;

#define LMCACHE_GPU_AESGCM_BATCH_FAULT_OFFSET 28

/* Workspace bytes for a batch of `count` objects; 0 when count > 2^20. */
size_t lmcache_gpu_aes128gcm_batch_workspace_size(size_t count);

int lmcache_gpu_aes128gcm_seal_batch_async(lmcache_gpu_aesgcm_key_t key, lmcache_gpu_aesgcm_batch_item* items,
                                           size_t count, void* workspace, size_t workspace_bytes,
                                           void* stream);

int lmcache_gpu_aes128gcm_open_batch_async(lmcache_gpu_aesgcm_key_t key, lmcache_gpu_aesgcm_batch_item* items,
                                           size_t count, void* workspace, size_t workspace_bytes,
                                           void* stream);

/* rc -> static string (reference gpu_aesgcm_api.h:90-92). */
const char* lmcache_gpu_aesgcm_strerror(int rc);

#ifdef __cplusplus
}
#endif
