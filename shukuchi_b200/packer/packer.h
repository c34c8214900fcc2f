/* packer.h -- GGUF -> LSTR container packer (model_packer/include/packer.h of
 * the reference: the same config struct and entry point; the reference's
 * packer_run is an empty stub). */
#ifndef SHK_PACKER_H
#define SHK_PACKER_H

#include <stdint.h>

struct packer_config {
    int prefer_gguf;         /* input is GGUF (the only input format) */
    uint32_t alignment;      /* layer-block alignment: 4096 (default) or 2 MiB */
    int write_checksums;     /* XXH64 of every layer block in the index */
};

/* 0 on success, -1 on a read / format / write error. */
int packer_run(const char *input_path, const char *output_path, const struct packer_config *cfg);

#endif
