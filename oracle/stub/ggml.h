/*
 * Minimal stand-in for <ggml.h> -- TEST INFRASTRUCTURE ONLY.
 *
 * zonos2_model.cpp includes <ggml.h> but only touches ggml_tensor's data and
 * view_offs fields (src/zonos2_model.cpp:11-13), in a helper nothing calls;
 * the ggml_context parameter of zonos2_forward is unused (:628).  ggml itself
 * is not installed here, so the reference's sources compile against this.
 */
#pragma once
#include <cstddef>

struct ggml_context;
struct ggml_cgraph;
struct ggml_tensor {
    void *data;
    size_t view_offs;
};
