/* main.c -- packer CLI (model_packer/src/main.c): shukuchi-pack <input.gguf>
 * <output.lstr> [--align N] [--checksums].  Defaults as the reference's main:
 * 4096-byte layer alignment, no checksums. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "packer.h"

int main(int argc, char **argv) {
    if (argc < 3) {
        fprintf(stderr, "Usage: %s <input> <output> [--align N] [--checksums]\n", argv[0]);
        return 1;
    }
    struct packer_config cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.prefer_gguf = 1;
    cfg.alignment = 4096;
    cfg.write_checksums = 0;
    for (int i = 3; i < argc; ++i) {
        if (strcmp(argv[i], "--align") == 0 && i + 1 < argc) cfg.alignment = (uint32_t)strtoul(argv[++i], NULL, 10);
        else if (strcmp(argv[i], "--checksums") == 0) cfg.write_checksums = 1;
    }
    const int rc = packer_run(argv[1], argv[2], &cfg);
    if (rc) fprintf(stderr, "packer: failed\n");
    return rc ? 1 : 0;
}
