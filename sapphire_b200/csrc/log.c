// log.c - leveled stderr logger for libsapphire_cuda.so.
//
// Same levels and environment switch as the reference logger
// (src/log.c:46-66): SAPPHIRE_LOG_LEVEL = debug | info | warn | error | none
// or a number.  The default is "warn" so a library call that succeeds is
// silent; every failing entry point logs one ERROR line.
#define _POSIX_C_SOURCE 200809L
#include <ctype.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#include "common.h"

static int g_level = -1;
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static void read_env_level(void) {
    int level = SAPPHIRE_LOG_WARN;
    const char *v = getenv("SAPPHIRE_LOG_LEVEL");
    if (v && *v) {
        char buf[16];
        size_t n = 0;
        while (*v && n + 1 < sizeof buf) buf[n++] = (char)tolower((unsigned char)*v++);
        buf[n] = 0;
        if (!strcmp(buf, "debug")) level = SAPPHIRE_LOG_DEBUG;
        else if (!strcmp(buf, "info")) level = SAPPHIRE_LOG_INFO;
        else if (!strcmp(buf, "warn") || !strcmp(buf, "warning")) level = SAPPHIRE_LOG_WARN;
        else if (!strcmp(buf, "error")) level = SAPPHIRE_LOG_ERROR;
        else if (!strcmp(buf, "none")) level = SAPPHIRE_LOG_NONE;
        else {
            char *end = NULL;
            long lv = strtol(buf, &end, 10);
            if (end && end != buf) level = (int)lv;
        }
    }
    g_level = level;
}

void sapphire_log(int level, const char *file, int line, const char *func, const char *fmt, ...) {
    pthread_once(&g_once, read_env_level);
    if (level < g_level) return;
    const char *tag = level >= SAPPHIRE_LOG_ERROR ? "ERROR"
                    : level >= SAPPHIRE_LOG_WARN  ? "WARN"
                    : level >= SAPPHIRE_LOG_INFO  ? "INFO" : "DEBUG";
    const char *base = strrchr(file, '/');
    base = base ? base + 1 : file;
    char msg[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    fprintf(stderr, "[sapphire %s] %s:%d %s: %s\n", tag, base, line, func, msg);
}
