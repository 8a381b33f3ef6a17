/* Test driver: the reference's native service generator (service/native.c,
 * compiled unchanged from the reference's sources, with a SHA-256 stand-in for
 * Apple's CommonCrypto header) driving liblunelette_cuda.so through
 * include/metal.h on Linux, over multi-turn sessions of token ids:
 *
 *   service_native_turns CHECKPOINT IDS_FILE PREFIX TURNS USER GENERATE
 *
 * IDS_FILE holds PREFIX system ids, then TURNS x USER user ids. The driver
 * opens the generator with prefix reuse on at context 4352 (blocks of 256),
 * materializes the prefix and saves it, then runs each turn the way the
 * service's session worker does: materialize the history plus the user ids
 * (prefilled as appends after the reused prefix), take GENERATE greedy ids
 * with next(), materializing each one before the next (a decode). The
 * checkpoint is saved at the last turn's user ids; at the end the driver
 * restores it and generates that turn's ids again. Output:
 *   turn <t>: <ids>      ttft_ms <t>: <ms>      replay: <ids>
 * The tokenizer is the reference's synthetic Tekken fixture
 * (tests/support/tokenizer_fixture.h), written into the working directory;
 * only token ids cross the generator here. */
#include "native.h"

#include "support/tokenizer_fixture.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now_ms(void)
{
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec * 1e3 + t.tv_nsec / 1e6;
}

/* Materialize seq[0..length) block by block; 1 when ready. */
static int materialize_all(service_generator *g, const unsigned *seq, unsigned length)
{
    for (int rounds = 0; rounds < 64; rounds++) {
        int r = g->materialize(g->context, seq, length);
        if (r == SERVICE_MATERIALIZE_READY) {
            return 1;
        }
        if (r != SERVICE_MATERIALIZE_MORE) {
            return 0;
        }
    }
    return 0;
}

/* GENERATE greedy ids after a materialized prompt of `length` ids in seq;
 * every id but the last is materialized (decoded) before the next one. */
static int generate(service_generator *g, unsigned *seq, unsigned *length, unsigned count, unsigned *out)
{
    for (unsigned i = 0; i < count; i++) {
        int id = g->next(g->context);
        if (id < 0) {
            return 0;
        }
        out[i] = (unsigned)id;
        seq[(*length)++] = (unsigned)id;
        if (i + 1 < count && !materialize_all(g, seq, *length)) {
            return 0;
        }
    }
    return 1;
}

int main(int argc, char **argv)
{
    if (argc != 7) {
        fputs("usage: service_native_turns CHECKPOINT IDS_FILE PREFIX TURNS USER GENERATE\n", stderr);
        return 2;
    }
    unsigned prefix = (unsigned)atoi(argv[3]), turns = (unsigned)atoi(argv[4]);
    unsigned user = (unsigned)atoi(argv[5]), gen = (unsigned)atoi(argv[6]);
    unsigned total = prefix + turns * (user + gen);
    if (!prefix || !turns || !user || !gen || total > SERVICE_CONTEXT_MAX) {
        fputs("sizes exceed the context\n", stderr);
        return 2;
    }
    unsigned *ids = malloc((size_t)(prefix + turns * user) * sizeof *ids);
    unsigned *seq = malloc((size_t)total * sizeof *seq);
    unsigned *saved = malloc((size_t)total * sizeof *saved);
    unsigned *out = malloc((size_t)gen * sizeof *out);
    FILE *in = fopen(argv[2], "r");
    if (!ids || !seq || !saved || !out || !in) {
        return 1;
    }
    for (unsigned i = 0; i < prefix + turns * user; i++) {
        if (fscanf(in, "%u", &ids[i]) != 1) {
            fputs("short ids file\n", stderr);
            return 1;
        }
    }
    fclose(in);
    synthetic_file(0);
    char *args[] = {"service", "--model", argv[1], "--tokenizer", (char *)scratch,
        "--strategy", "compact-fp8-arithmetic", "--prefill", "mps", "--context", "4352",
        "--prefill-chunk", "256", "--prefix-reuse", "on", "--port", "0"};
    service_generator g;
    unsigned port = 1;
    if (!service_native_open((int)(sizeof args / sizeof *args), args, &g, &port)) {
        fputs("service_native_open failed\n", stderr);
        return 1;
    }
    int ok = 1;
    unsigned length = 0, saved_length = 0;
    for (unsigned i = 0; i < prefix; i++) {
        seq[length++] = ids[i];
    }
    ok = materialize_all(&g, seq, length) && g.save(g.context) == 1;
    for (unsigned t = 0; ok && t < turns; t++) {
        double start = now_ms();
        for (unsigned i = 0; i < user; i++) {
            seq[length++] = ids[prefix + t * user + i];
        }
        ok = materialize_all(&g, seq, length);
        if (ok && t + 1 == turns) {
            ok = g.save(g.context) == 1;
            memcpy(saved, seq, length * sizeof *seq);
            saved_length = length;
        }
        double ttft = 0;
        if (ok) {
            int first = g.next(g.context);
            ttft = now_ms() - start;
            ok = first >= 0;
            if (ok) {
                out[0] = (unsigned)first;
                seq[length++] = (unsigned)first;
                ok = gen == 1 || (materialize_all(&g, seq, length) &&
                    generate(&g, seq, &length, gen - 1, out + 1));
            }
        }
        if (ok) {
            printf("turn %u:", t);
            for (unsigned i = 0; i < gen; i++) {
                printf(" %u", out[i]);
            }
            printf("\nttft_ms %u: %.3f\n", t, ttft);
        }
    }
    if (ok) {
        /* back to the saved last user prompt: the same ids again */
        ok = g.restore(g.context) == 1;
        length = saved_length;
        memcpy(seq, saved, length * sizeof *seq);
        ok = ok && generate(&g, seq, &length, gen, out);
        if (ok) {
            printf("replay:");
            for (unsigned i = 0; i < gen; i++) {
                printf(" %u", out[i]);
            }
            printf("\n");
        }
    }
    g.destroy(g.context);
    remove(scratch);
    free(ids);
    free(seq);
    free(saved);
    free(out);
    if (!ok) {
        fputs("service turn failed\n", stderr);
    }
    return ok ? 0 : 1;
}
