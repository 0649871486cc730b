/**
 * @file debug.hpp
 * @brief Logging macros with the reference's names (utils/debug.hpp:71-129),
 *        active when CHOREO_IR_DEBUG is defined.
 */
#ifndef CHOREO_IR_UTILS_DEBUG_HPP
#define CHOREO_IR_UTILS_DEBUG_HPP

#include <cstdio>
#include <stdexcept>

#include "../core/config.hpp"

#define CHOREO_LOG_(level, ...)                         \
  do {                                                  \
    if (::choreo_ir::config::DEBUG_MODE) {              \
      std::fprintf(stderr, "[choreo-ir %s] ", level);   \
      std::fprintf(stderr, __VA_ARGS__);                \
      std::fprintf(stderr, "\n");                       \
    }                                                   \
  } while (0)
#define CHOREO_DEBUG(...) CHOREO_LOG_("DEBUG", __VA_ARGS__)
#define CHOREO_INFO(...) CHOREO_LOG_("INFO", __VA_ARGS__)
#define CHOREO_WARNING(...) CHOREO_LOG_("WARNING", __VA_ARGS__)
#define CHOREO_ERROR(...) CHOREO_LOG_("ERROR", __VA_ARGS__)
#define CHOREO_ASSERT(cond, msg)                                                   \
  do {                                                                             \
    if (::choreo_ir::config::ENABLE_ASSERTIONS && !(cond)) throw std::runtime_error(msg); \
  } while (0)

#endif  // CHOREO_IR_UTILS_DEBUG_HPP
