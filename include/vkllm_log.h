/* Minimal leveled logger standing in for rxi/log.c, which the reference logs through
 * (thirdparty/log.c/repo.bzl:3-9). Same macro names: log_trace/debug/info/warn/error/fatal.
 * The level is read once from the environment variable VKLLM_LOG_LEVEL (0=trace .. 5=fatal, default 3=warn). */
#ifndef VKLLM_LOG_H
#define VKLLM_LOG_H

#ifdef __cplusplus
extern "C" {
#endif

enum
{
    VKLLM_LOG_TRACE = 0,
    VKLLM_LOG_DEBUG,
    VKLLM_LOG_INFO,
    VKLLM_LOG_WARN,
    VKLLM_LOG_ERROR,
    VKLLM_LOG_FATAL
};

extern void vkllm_log(int level, const char *file, int line, const char *fmt, ...)
#if defined(__GNUC__)
    __attribute__((format(printf, 4, 5)))
#endif
    ;
extern void vkllm_log_set_level(int level);

#ifndef log_error
#define log_trace(...) vkllm_log(VKLLM_LOG_TRACE, __FILE__, __LINE__, __VA_ARGS__)
#define log_debug(...) vkllm_log(VKLLM_LOG_DEBUG, __FILE__, __LINE__, __VA_ARGS__)
#define log_info(...) vkllm_log(VKLLM_LOG_INFO, __FILE__, __LINE__, __VA_ARGS__)
#define log_warn(...) vkllm_log(VKLLM_LOG_WARN, __FILE__, __LINE__, __VA_ARGS__)
#define log_error(...) vkllm_log(VKLLM_LOG_ERROR, __FILE__, __LINE__, __VA_ARGS__)
#define log_fatal(...) vkllm_log(VKLLM_LOG_FATAL, __FILE__, __LINE__, __VA_ARGS__)
#endif

#ifdef __cplusplus
}
#endif
#endif
