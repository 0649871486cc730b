/**
 * @file compute_impl.hpp
 * @brief Kept so code that includes the reference's compute_impl.hpp still
 *        compiles; the definitions live in matmul.hpp.
 */
#ifndef CHOREO_IR_COMPUTE_COMPUTE_IMPL_HPP
#define CHOREO_IR_COMPUTE_COMPUTE_IMPL_HPP
#include "compute.hpp"
#include "matmul.hpp"
#endif  // CHOREO_IR_COMPUTE_COMPUTE_IMPL_HPP
