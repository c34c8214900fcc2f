/* main.c -- engine CLI with the reference's flags (engine/src/main.c:28-109):
 *   shukuchi <model.gguf> [--prompt "..."] [--max-tokens N] [--tokens 1,2,3]
 * SHUKUCHI_PREFETCH_DEPTH sets the loader depth (default 3; 0 -> 2).  Tokens
 * are printed as "<id>text"; the streaming statistics line follows on stderr.
 * --tokens (an addition) feeds token ids instead of prompt text. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/resource.h>

#include "engine.h"

int main(int argc, char **argv) {
    if (argc < 2) {
        fprintf(stderr, "Usage: %s <model.gguf> [--prompt \"...\"] [--max-tokens N] [--tokens 1,2,3]\n", argv[0]);
        return 1;
    }
    uint32_t max_tokens = 16;
    const char *prompt = NULL, *tokens = NULL;
    for (int i = 2; i + 1 < argc; ++i) {
        if (strcmp(argv[i], "--max-tokens") == 0) max_tokens = (uint32_t)strtoul(argv[++i], NULL, 10);
        else if (strcmp(argv[i], "--prompt") == 0) prompt = argv[++i];
        else if (strcmp(argv[i], "--tokens") == 0) tokens = argv[++i];
    }
    uint32_t depth = 3;
    const char *env = getenv("SHUKUCHI_PREFETCH_DEPTH");
    if (env && *env) {
        depth = (uint32_t)strtoul(env, NULL, 10);
        if (depth == 0) depth = 2;
    }
    struct engine_config cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.n_threads = 4;
    cfg.batch_size = 1;
    cfg.prefetch_depth = depth;
    cfg.kv_block_size = 32;
    engine_handle_t *h = engine_open(argv[1], &cfg);
    if (!h) {
        fprintf(stderr, "engine: failed to open model\n");
        return 1;
    }
    int rc;
    if (tokens) {
        uint32_t ids[4096];
        uint32_t n = 0;
        for (const char *p = tokens; *p && n < 4096;) {
            char *end;
            ids[n++] = (uint32_t)strtoul(p, &end, 10);
            p = (*end == ',') ? end + 1 : end;
            if (end == p && *p) break;
        }
        rc = engine_generate_ids(h, ids, n, max_tokens, NULL, NULL) < 0;
        if (!rc) printf("%s\n", engine_get_output(h));
    } else {
        if (prompt) engine_set_prompt(h, prompt);
        rc = engine_generate(h, max_tokens) != 0;
    }
    struct streaming_stats st;
    if (engine_get_streaming_stats(h, &st) == 0)
        fprintf(stderr,
                "streaming_stats: layer_loads=%llu layer_bytes_read=%llu max_layer_size=%zu peak_buffer_usage=%zu "
                "peak_rss=%zu max_concurrent_buffers=%u prefetch_hits=%u prefetch_misses=%u\n",
                (unsigned long long)st.layer_loads, (unsigned long long)st.layer_bytes_read, st.max_layer_size,
                st.peak_buffer_usage, st.peak_rss, st.max_concurrent_buffers, st.prefetch_hits,
                st.prefetch_misses);
    engine_report(h); /* engine/src/main.c:106 metal_ops_report() */
    engine_close(h);
    struct rusage ru;
    if (getrusage(RUSAGE_SELF, &ru) == 0) fprintf(stderr, "peak_rss_mb=%.2f\n", (double)ru.ru_maxrss / 1024.0);
    if (rc) fprintf(stderr, "engine: generation failed\n");
    return rc;
}
