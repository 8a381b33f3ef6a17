/* SHA-256 (FIPS 180-4) under the names the reference's service/native.c
 * includes from Apple's CommonCrypto (<CommonCrypto/CommonDigest.h>), so that
 * file compiles unchanged on Linux. Only what native.c uses is provided:
 * CC_SHA256_CTX, CC_SHA256_Init/Update/Final, CC_SHA256_DIGEST_LENGTH and
 * CC_LONG. Header-only; written from the standard's description (message
 * schedule, 64 rounds over eight 32-bit working variables, big-endian length
 * padding). Test support only: the service uses it to fingerprint the model
 * and tokenizer files it reports. */
#ifndef LUNELETTE_COMMONCRYPTO_SHIM_H
#define LUNELETTE_COMMONCRYPTO_SHIM_H

#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define CC_SHA256_DIGEST_LENGTH 32
typedef uint32_t CC_LONG;

typedef struct {
    uint32_t state[8];
    uint64_t bits;          /* message length so far, in bits */
    unsigned char block[64];
    size_t used;            /* bytes waiting in block */
} CC_SHA256_CTX;

/* Round constants: the first 32 bits of the fractional parts of the cube
 * roots of the first 64 primes (FIPS 180-4, 4.2.2). */
static const uint32_t lun_sha256_k[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

static inline uint32_t lun_rotr(uint32_t x, unsigned n) { return (x >> n) | (x << (32 - n)); }

static inline void lun_sha256_block(uint32_t state[8], const unsigned char *p)
{
    uint32_t w[64];
    for (int i = 0; i < 16; i++) {
        w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 |
            (uint32_t)p[4 * i + 3];
    }
    for (int i = 16; i < 64; i++) {
        uint32_t s0 = lun_rotr(w[i - 15], 7) ^ lun_rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = lun_rotr(w[i - 2], 17) ^ lun_rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = state[0], b = state[1], c = state[2], d = state[3];
    uint32_t e = state[4], f = state[5], g = state[6], h = state[7];
    for (int i = 0; i < 64; i++) {
        uint32_t big1 = lun_rotr(e, 6) ^ lun_rotr(e, 11) ^ lun_rotr(e, 25);
        uint32_t choose = (e & f) ^ (~e & g);
        uint32_t t1 = h + big1 + choose + lun_sha256_k[i] + w[i];
        uint32_t big0 = lun_rotr(a, 2) ^ lun_rotr(a, 13) ^ lun_rotr(a, 22);
        uint32_t majority = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = big0 + majority;
        h = g;
        g = f;
        f = e;
        e = d + t1;
        d = c;
        c = b;
        b = a;
        a = t1 + t2;
    }
    state[0] += a;
    state[1] += b;
    state[2] += c;
    state[3] += d;
    state[4] += e;
    state[5] += f;
    state[6] += g;
    state[7] += h;
}

static inline int CC_SHA256_Init(CC_SHA256_CTX *ctx)
{
    /* initial hash value: fractional parts of the square roots of the first
     * eight primes (FIPS 180-4, 5.3.3) */
    static const uint32_t h0[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                                   0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    memcpy(ctx->state, h0, sizeof h0);
    ctx->bits = 0;
    ctx->used = 0;
    return 1;
}

static inline int CC_SHA256_Update(CC_SHA256_CTX *ctx, const void *data, CC_LONG length)
{
    const unsigned char *p = data;
    ctx->bits += (uint64_t)length * 8;
    while (length) {
        if (ctx->used == 0 && length >= 64) {
            lun_sha256_block(ctx->state, p);
            p += 64;
            length -= 64;
            continue;
        }
        size_t take = 64 - ctx->used < length ? 64 - ctx->used : length;
        memcpy(ctx->block + ctx->used, p, take);
        ctx->used += take;
        p += take;
        length -= (CC_LONG)take;
        if (ctx->used == 64) {
            lun_sha256_block(ctx->state, ctx->block);
            ctx->used = 0;
        }
    }
    return 1;
}

static inline int CC_SHA256_Final(unsigned char *digest, CC_SHA256_CTX *ctx)
{
    uint64_t bits = ctx->bits;
    ctx->block[ctx->used++] = 0x80;
    if (ctx->used > 56) {
        memset(ctx->block + ctx->used, 0, 64 - ctx->used);
        lun_sha256_block(ctx->state, ctx->block);
        ctx->used = 0;
    }
    memset(ctx->block + ctx->used, 0, 56 - ctx->used);
    for (int i = 0; i < 8; i++) {
        ctx->block[56 + i] = (unsigned char)(bits >> (56 - 8 * i));
    }
    lun_sha256_block(ctx->state, ctx->block);
    for (int i = 0; i < 8; i++) {
        digest[4 * i] = (unsigned char)(ctx->state[i] >> 24);
        digest[4 * i + 1] = (unsigned char)(ctx->state[i] >> 16);
        digest[4 * i + 2] = (unsigned char)(ctx->state[i] >> 8);
        digest[4 * i + 3] = (unsigned char)ctx->state[i];
    }
    return 1;
}

#endif
