#include "log.h"

#include <stdarg.h>
#include <stdlib.h>
#include <time.h>

static int g_level = -1;

int cc_log_level(void)
{
    int lvl = __atomic_load_n(&g_level, __ATOMIC_RELAXED);
    if (lvl < 0) {
        const char *s = getenv("CROSSCACHE_LOG");
        lvl = s ? atoi(s) : 1;
        __atomic_store_n(&g_level, lvl, __ATOMIC_RELAXED);
    }
    return lvl;
}

void cc_log_write(int level, const char *file, int line, const char *fmt, ...)
{
    static const char *names[] = {"FATAL", "ERROR", "WARN", "INFO", "DEBUG"};
    char msg[1024];
    struct timespec ts;
    va_list ap;

    va_start(ap, fmt);
    vsnprintf(msg, sizeof(msg), fmt, ap);
    va_end(ap);
    clock_gettime(CLOCK_REALTIME, &ts);
    fprintf(stderr, "[crosscache %ld.%06ld %s %s:%d] %s\n", (long)ts.tv_sec,
            ts.tv_nsec / 1000, names[level < 0 ? 0 : (level > 4 ? 4 : level)],
            file, line, msg);
}
