/* ORACLE build shim: no-op stand-in for the log.h of CrossCache's absent
 * infrastructure submodule, so that the reference's own
 * src/device/mem/mem.cpp compiles unchanged for oracle/_ref. */
#ifndef ORACLE_REFSHIM_LOG_H
#define ORACLE_REFSHIM_LOG_H
#define log_fatal(...) ((void)0)
#define log_error(...) ((void)0)
#define log_warn(...) ((void)0)
#define log_info(...) ((void)0)
#define log_debug(...) ((void)0)
#endif
