/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * OpenSSL EVP AES-128-GCM seal with a caller-supplied IV. It makes the same
 * EVP calls in the same order as the reference's native backend
 * (experiments/gpu_kv_seal/native/cpu_seal_openssl.cpp:140-206: EncryptInit
 * with the cipher, SET_IVLEN 12, EncryptInit with key and IV, Update over the
 * plaintext, Final, GET_TAG 16) and writes the same frame
 * [1 | IV | ciphertext | tag]. The reference draws its IV from RAND_bytes
 * (cpu_seal_openssl.cpp:146-148), so byte-exact frames for a seeded IV need
 * this injected-IV variant. The reference's own open
 * (lmcache_aes128gcm_open) is used unchanged from oracle/_ref.
 *
 * Thread-safe: each call owns its EVP context.
 */
#include <limits.h>
#include <stddef.h>
#include <stdint.h>

#include <openssl/evp.h>

int oracle_evp_seal_iv(const uint8_t* key, const uint8_t* iv, const uint8_t* src, size_t len,
                       uint8_t* frame, size_t frame_cap)
{
    if (key == NULL || iv == NULL || frame == NULL || (src == NULL && len != 0)) {
        return -1;
    }
    if (frame_cap < len + 29u) {
        return -2;
    }
    EVP_CIPHER_CTX* ctx = EVP_CIPHER_CTX_new();
    if (ctx == NULL) {
        return -3;
    }
    int rc = 0;
    frame[0] = 1;
    for (int i = 0; i < 12; ++i) {
        frame[1 + i] = iv[i];
    }
    uint8_t* ct = frame + 13;
    if (EVP_EncryptInit_ex(ctx, EVP_aes_128_gcm(), NULL, NULL, NULL) != 1 ||
        EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_SET_IVLEN, 12, NULL) != 1 ||
        EVP_EncryptInit_ex(ctx, NULL, NULL, key, iv) != 1) {
        rc = -4;
        goto done;
    }
    size_t done_len = 0;
    while (done_len < len) {
        const size_t remain = len - done_len;
        const int chunk = remain > (size_t)INT_MAX ? INT_MAX : (int)remain;
        int produced = 0;
        if (EVP_EncryptUpdate(ctx, ct + done_len, &produced, src + done_len, chunk) != 1 ||
            produced != chunk) {
            rc = -5;
            goto done;
        }
        done_len += (size_t)chunk;
    }
    int final_len = 0;
    if (EVP_EncryptFinal_ex(ctx, ct + len, &final_len) != 1 || final_len != 0) {
        rc = -6;
        goto done;
    }
    if (EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_GET_TAG, 16, ct + len) != 1) {
        rc = -7;
        goto done;
    }
done:
    EVP_CIPHER_CTX_free(ctx);
    return rc;
}
