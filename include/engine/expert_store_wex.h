/* The WEX expert-store backend of the engine (the reference's c/expert_store_wex.h:24-29), kept as an
 * interface only: this library does not implement it.
 *
 * The store (its slab cache, leases, LRU and miss reads: the reference's c/expert_store_wex.c) belongs to
 * the engine and is built there, against the engine's own expert_store.h and deepseek_v4_internal.h,
 * which this header takes from the engine's include path as the reference's header does. The store
 * decodes every miss through the engine API of ../wex_decode.h (coli_wex_decode_record), which this
 * library implements on the GPU, so the store links against this library unchanged. A store that wants
 * the whole miss path on the GPU (reads into page-locked memory, uploads and decodes overlapped) calls
 * wexb_file_decode of ../wexb200.h from its miss handler in place of its pread and decode. */
#ifndef WEXB_EXPERT_STORE_WEX_H
#define WEXB_EXPERT_STORE_WEX_H
#include <stddef.h>

#include "deepseek_v4_internal.h" /* engine: ColiV4Engine, ColiDeepSeekV4Config, ColiDeepSeekV4ExpertStoreOptions */
#include "expert_store.h"         /* engine: ColiExpertStore */
#include "../wex_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Registered under the name "wex" in the engine's store registry: opens the engine's legacy expert
 * container (options->model_dir when it names a .wex file, else v4_flash_experts.wex inside it) and
 * returns the store in *output, or a non-zero status with a message in error. */
int coli_v4_expert_store_open_wex(ColiV4Engine *engine, const ColiDeepSeekV4Config *config,
                                  const ColiDeepSeekV4ExpertStoreOptions *options, ColiExpertStore **output,
                                  char *error, size_t error_size);

#ifdef __cplusplus
}
#endif
#endif
