/* Test infrastructure: drives llama98-zh_b200/shim/lz98_gpu_shim.c.
     shim_main SO accept
         model-free acceptance through the shim (host only, no GPU);
     shim_main SO generate MODEL_DIR K TEMP SEED N_ROUNDS TOKEN...
         the reference loop's prefill and N_ROUNDS speculative rounds of
         depth K through the shim; prints every emitted token. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "lz98_gpu.h"
#include "lz98_gpu_shim.h"

static int accept_cases(void) {
    int draft[3] = {5, 7, 9}, targ[3] = {5, 7, 1}, out[4] = {0}, n;
    float p[4] = {0.1f, 0.6f, 0.2f, 0.1f}, q[4] = {0.4f, 0.2f, 0.2f, 0.2f};
    uint64_t rng = 42;
    int acc = -1, tok;
    n = gpu_spec_accept(draft, targ, 3, 11, out);
    printf("accept %d %d %d %d\n", n, out[0], out[1], out[2]);
    targ[2] = 9;
    n = gpu_spec_accept(draft, targ, 3, 11, out);
    printf("accept %d %d %d %d %d\n", n, out[0], out[1], out[2], out[3]);
    tok = gpu_spec_accept_temp(p, q, 1, 4, 0.3f, &rng, &acc);
    printf("temp %d %d\n", tok, acc);
    tok = gpu_spec_accept_temp(p, q, 0, 4, 0.9f, &rng, &acc);
    printf("temp %d %d %llu\n", tok, acc, (unsigned long long)rng);
    return 0;
}

int main(int argc, char **argv) {
    char err[256] = "";
    if (argc < 3) return 2;
    if (gpu_load(argv[1], err, sizeof err)) { fprintf(stderr, "%s\n", err); return 1; }
    if (!strcmp(argv[2], "accept")) return accept_cases();
    if (!strcmp(argv[2], "generate") && argc > 8) {
        const int k = atoi(argv[4]), n_rounds = atoi(argv[7]), n_prompt = argc - 8;
        int *prompt = malloc(sizeof(int) * (size_t)n_prompt), i, r, anchor = 0, pos, rc;
        LZSampler samp;
        memset(&samp, 0, sizeof samp);
        samp.p.temperature = (float)atof(argv[5]);
        samp.p.topp = 0.95f;
        samp.p.repetition_penalty = 1.0f;
        samp.rng_state = strtoull(argv[6], NULL, 10);
        for (i = 0; i < n_prompt; i++) prompt[i] = atoi(argv[8 + i]);
        if (gpu_open(argv[3], n_prompt + 8 * n_rounds + 64, k, err, sizeof err)) {
            fprintf(stderr, "%s\n", err);
            return 1;
        }
        if (gpu_prefill(prompt, n_prompt, &samp, &anchor, err, sizeof err)) {
            fprintf(stderr, "%s\n", err);
            return 1;
        }
        printf("%d", anchor);
        pos = n_prompt - 1;   /* anchor_pos: the last forwarded position */
        for (r = 0; r < n_rounds; r++) {
            int out[8], na = 0, np = 0, ke = 0;
            rc = gpu_spec_round(anchor, pos, k, 0.0f, 0, &samp, out, &na, &np, &ke, err, sizeof err);
            if (rc < 0) { fprintf(stderr, "%s\n", err); return 1; }
            for (i = 0; i <= na; i++) printf(" %d", out[i]);
            anchor = out[na];
            pos = np;
        }
        printf("\n");
        gpu_close();
        free(prompt);
        return 0;
    }
    return 2;
}
