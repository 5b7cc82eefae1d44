// The C ABI's opaque handle for synchronous inference, shared by the files
// that implement entry points on it.
#pragma once
#include <memory>

#include "engine.hpp"

struct azb_infer {
    std::unique_ptr<azb::Inference> impl;
};
