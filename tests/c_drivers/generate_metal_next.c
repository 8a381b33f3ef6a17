/* Test driver: the reference's own greedy generation loop (src/generation.c,
 * compiled from the reference's sources with its include/ headers) driving
 * liblunelette_cuda.so through the include/metal.h contract, unchanged. The
 * logits callback does what the reference's CLI callback does
 * (src/main.c:48-67): the first call prefills the whole prompt, every later
 * call decodes the newest id, and the borrowed logits are copied into the
 * loop's buffer.
 *
 *   generate_metal_next CHECKPOINT MAX_NEW_TOKENS ID [ID ...]
 *
 * Prints "tokens: <id> ..." and "stop: <reason>" (0 limit, 1 EOS, 2 context)
 * on success; exits 1 with the runtime's diagnostic otherwise. */
#include "generation.h"
#include "metal.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    lunelette_metal *context;
    int prefilled;
    size_t calls;
} next_state;

static int next_logits(void *opaque, const int64_t *ids, size_t count, float *logits, char *error,
    size_t capacity)
{
    next_state *state = opaque;
    const float *borrowed = NULL;
    int status = state->prefilled ?
        lunelette_metal_decode(state->context, ids[count - 1], &borrowed, error, capacity) :
        lunelette_metal_prefill(state->context, ids, count, &borrowed, error, capacity);
    if (status != 0) {
        return -1;
    }
    state->prefilled = 1;
    state->calls++;
    memcpy(logits, borrowed, LUNELETTE_VOCAB_SIZE * sizeof(float));
    return 0;
}

int main(int argc, char **argv)
{
    if (argc < 4) {
        fputs("usage: generate_metal_next CHECKPOINT MAX_NEW_TOKENS ID [ID ...]\n", stderr);
        return 2;
    }
    size_t count = (size_t)(argc - 3);
    int64_t *prompt = malloc(count * sizeof *prompt);
    if (!prompt) {
        return 1;
    }
    for (size_t i = 0; i < count; i++) {
        prompt[i] = strtoll(argv[3 + i], NULL, 10);
    }
    char error[512] = "";
    lunelette_metal *context = lunelette_metal_create(argv[1], error, sizeof error);
    if (!context) {
        fprintf(stderr, "create: %s\n", error);
        free(prompt);
        return 1;
    }
    lunelette_generation_config config = LUNELETTE_GENERATION_DEFAULT;
    config.max_new_tokens = (size_t)strtoul(argv[2], NULL, 10);
    lunelette_generation_result result;
    next_state state = {context, 0, 0};
    int status = lunelette_generate_with_logits(next_logits, &state, prompt, count, &config, &result,
        error, sizeof error);
    if (status != 0) {
        fprintf(stderr, "generate: %s\n", error);
    } else {
        printf("tokens:");
        for (size_t i = 0; i < result.count; i++) {
            printf(" %lld", (long long)result.tokens[i]);
        }
        printf("\nstop: %d\ncalls: %zu\n", (int)result.stop, state.calls);
    }
    lunelette_metal_destroy(context);
    free(prompt);
    return status ? 1 : 0;
}
