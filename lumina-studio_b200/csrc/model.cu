// Decode model: placeholder entries until the model runtime lands.
#include "common.cuh"

using namespace lumina;

#define NOT_YET(fn)                                   \
  do {                                                \
    set_error("%s: not implemented in this build", fn); \
    return LUMINA_E_UNSUPPORTED;                      \
  } while (0)

extern "C" {
int lumina_model_create(int, const lumina_model_config*, lumina_model**) { NOT_YET("model_create"); }
int lumina_model_set_weight(lumina_model*, const char*, lumina_weight*) { NOT_YET("model_set_weight"); }
int lumina_model_set_tensor(lumina_model*, const char*, const float*, int, int) { NOT_YET("model_set_tensor"); }
int lumina_model_finalize(lumina_model*) { NOT_YET("model_finalize"); }
int lumina_model_free(lumina_model*) { return LUMINA_OK; }
int lumina_nccl_unique_id(uint8_t*) { NOT_YET("nccl_unique_id"); }
int lumina_model_init_tp(lumina_model*, const uint8_t*) { NOT_YET("model_init_tp"); }
int lumina_kv_length(const lumina_model*, int*) { NOT_YET("kv_length"); }
int lumina_kv_truncate(lumina_model*, int) { NOT_YET("kv_truncate"); }
int lumina_kv_read(const lumina_model*, int, int, int, float*, float*) { NOT_YET("kv_read"); }
int lumina_kv_commit_rows(lumina_model*, int, const int*, int) { NOT_YET("kv_commit_rows"); }
int lumina_layer_forward(lumina_model*, int, float*, int, int, const int*, const float*, void*) { NOT_YET("layer_forward"); }
int lumina_forward(lumina_model*, const int*, int, int, float*, int) { NOT_YET("forward"); }
int lumina_decode_step(lumina_model*, int, float*, int*) { NOT_YET("decode_step"); }
}
