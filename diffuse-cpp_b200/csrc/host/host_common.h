// Logging and error plumbing of the host library.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <string>

namespace dfh {

// Same prefix and fatal behaviour as the reference's DIFFUSE_LOG / DIFFUSE_DIE
// (src/diffuse-common.h:17-21).  DIFFUSE_LOG_LEVEL=0 silences the informational lines.
bool log_enabled();
#define DIFFUSE_LOG(fmt, ...) \
    do { if (::dfh::log_enabled()) fprintf(stderr, "[diffuse] " fmt "\n", ##__VA_ARGS__); } while (0)
#define DIFFUSE_DIE(fmt, ...)                                          \
    do {                                                               \
        fprintf(stderr, "[diffuse] FATAL: " fmt "\n", ##__VA_ARGS__); \
        exit(1);                                                       \
    } while (0)

int set_error(int code, const char *fmt, ...);
const char *last_error();

bool quantize_rows(int type, const float *x, int64_t n, uint8_t *out);
bool dequantize_rows(int type, const uint8_t *src, int64_t n, float *dst);
int quantize_file(const char *in_path, const char *out_path, const char *type, int n_threads);

}  // namespace dfh
