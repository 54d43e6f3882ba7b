/* TEST INFRASTRUCTURE (oracle pin). The reference logs through rxi/log.c (thirdparty/log.c), which is
 * not vendored; its two macros that the reference's test files call print to stderr here. */
#ifndef REFPIN_STUB_LOG_H
#define REFPIN_STUB_LOG_H
#include <stdio.h>
#ifndef log_error
#define log_info(...) (fprintf(stderr, __VA_ARGS__), fputc('\n', stderr))
#define log_error(...) (fprintf(stderr, __VA_ARGS__), fputc('\n', stderr))
#define log_warn(...) (fprintf(stderr, __VA_ARGS__), fputc('\n', stderr))
#define log_debug(...) ((void)0)
#define log_trace(...) ((void)0)
#define log_fatal(...) (fprintf(stderr, __VA_ARGS__), fputc('\n', stderr))
#endif
#endif
