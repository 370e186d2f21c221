/* Test infrastructure only (never linked into the product library): drives
 * the C engine's own KV-cache persistence -- kvcache_save / kvcache_load,
 * picolm/model.c:870-983, compiled from the reference's sources -- on
 * caller-owned caches in its layout ([n_layers][max_seq_len][kv_dim] fp16),
 * so tests can compare the library's KVCP files with the reference's byte for
 * byte.  Only the fields those two functions read are filled in. */
#include <string.h>

#include "model.h"

static void fill(model_t* m, int n_layers, int n_kv_heads, int head_dim, int max_seq, uint16_t* kc, uint16_t* vc) {
    memset(m, 0, sizeof *m);
    m->config.n_layers = n_layers;
    m->config.n_kv_heads = n_kv_heads;
    m->config.head_dim = head_dim;
    m->config.max_seq_len = max_seq;
    m->state.key_cache = kc;
    m->state.val_cache = vc;
}

int pref_kvcp_save(int n_layers, int n_kv_heads, int head_dim, int max_seq, uint16_t* kc, uint16_t* vc,
                   const char* path, int n_pos) {
    model_t m;
    fill(&m, n_layers, n_kv_heads, head_dim, max_seq, kc, vc);
    return kvcache_save(&m, path, n_pos);
}

int pref_kvcp_load(int n_layers, int n_kv_heads, int head_dim, int max_seq, uint16_t* kc, uint16_t* vc,
                   const char* path) {
    model_t m;
    fill(&m, n_layers, n_kv_heads, head_dim, max_seq, kc, vc);
    return kvcache_load(&m, path);
}
