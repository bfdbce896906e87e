/*
 * Minimal leveled logger for the cache manager and adaptors.
 * Level from the environment variable CROSSCACHE_LOG
 * (0 = fatal, 1 = error (default), 2 = warn, 3 = info, 4 = debug).
 * Stands in for the zlog-backed log_* macros of CrossCache's absent
 * infrastructure submodule (call sites e.g. src/cache/cache.c:10).
 */
#ifndef CC_LOG_H
#define CC_LOG_H

#include <stdio.h>

#ifdef __cplusplus
extern "C" {
#endif

int cc_log_level(void);
void cc_log_write(int level, const char *file, int line, const char *fmt, ...)
    __attribute__((format(printf, 4, 5)));

#ifdef __cplusplus
}
#endif

#define CC_LOG(lvl, ...)                                                   \
    do {                                                                   \
        if (cc_log_level() >= (lvl))                                       \
            cc_log_write((lvl), __FILE__, __LINE__, __VA_ARGS__);          \
    } while (0)

#define log_fatal(...) CC_LOG(0, __VA_ARGS__)
#define log_error(...) CC_LOG(1, __VA_ARGS__)
#define log_warn(...)  CC_LOG(2, __VA_ARGS__)
#define log_info(...)  CC_LOG(3, __VA_ARGS__)
#define log_debug(...) CC_LOG(4, __VA_ARGS__)

#endif
