// medusa.h decode functions over the fl_engine.
#include "fl_common.cuh"
#include "fl_runtime.h"
#include "medusa.h"

using namespace fl;

FL_API int medusa_predict(medusa_model_t*, const float*, int, medusa_tree_t*, const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_predict: not available in this build"), -1;
}
FL_API int medusa_build_tree(medusa_model_t*, const float*, medusa_tree_t*, const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_build_tree: not available in this build"), -1;
}
FL_API int medusa_verify_tree(void*, void (*)(void*, const int*, int, float*, int), const medusa_tree_t*, int*, int*,
                              const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_verify_tree: not available in this build"), -1;
}
FL_API int medusa_decode_step(void*, void (*)(void*, const int*, int, float*, int), medusa_model_t*, const float*, int,
                              int*, int*, const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_decode_step: not available in this build"), -1;
}
FL_API int medusa_generate(void*, void (*)(void*, const int*, int, float*, int), medusa_model_t*, const float*, int,
                           int*, int, const medusa_config_t*) {
    return set_error(FL_E_UNSUPPORTED, "medusa_generate: not available in this build"), -1;
}
