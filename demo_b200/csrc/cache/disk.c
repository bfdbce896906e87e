/*
 * Disk tier file IO (see disk.h for the layout and the reference functions
 * it follows).
 */
#define _GNU_SOURCE
#include "disk.h"

#include "../infra/log.h"

#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <sys/types.h>
#include <unistd.h>

#define DIRECT_ALIGN 4096u

static uint64_t g_tmp_seq;

int disk_open_root(const char *root)
{
    int fd;

    if (!root || !*root)
        return -EINVAL;
    if (mkdir(root, S_IRWXU | S_IRGRP | S_IXGRP) && errno != EEXIST)
        return -errno;
    fd = open(root, O_RDONLY | O_DIRECTORY | O_CLOEXEC);
    return fd < 0 ? -errno : fd;
}

int disk_open_ns(int rootfd, const char *tag, uint8_t tp_size, uint8_t tp_id)
{
    char name[256];
    size_t i, n;
    int fd;

    n = strlen(tag);
    if (n > 200)
        n = 200;
    for (i = 0; i < n; i++) {
        char c = tag[i];
        name[i] = (c == '/' || c < 0x21 || c > 0x7e) ? '_' : c;
    }
    snprintf(name + n, sizeof(name) - n, ".tp%u.%u", tp_size, tp_id);
    if (!strcmp(name, ".") || !strcmp(name, ".."))
        return -EINVAL;
    if (mkdirat(rootfd, name, S_IRWXU | S_IRGRP | S_IXGRP) && errno != EEXIST)
        return -errno;
    fd = openat(rootfd, name, O_RDONLY | O_DIRECTORY | O_CLOEXEC);
    return fd < 0 ? -errno : fd;
}

void disk_key_name(const uint8_t *key, char name[DISK_NAME_LEN + 1])
{
    static const char hex[] = "0123456789abcdef";
    int i;

    for (i = 0; i < DISK_NAME_LEN / 2; i++) {
        name[2 * i] = hex[key[i] >> 4];
        name[2 * i + 1] = hex[key[i] & 15];
    }
    name[DISK_NAME_LEN] = '\0';
}

int disk_stat(int dfd, const uint8_t *key, uint64_t size)
{
    char name[DISK_NAME_LEN + 1];
    struct stat st;

    disk_key_name(key, name);
    if (fstatat(dfd, name, &st, 0) || !S_ISREG(st.st_mode) ||
        (uint64_t)st.st_size != size)
        return -ENOENT;
    return 0;
}

static int direct_ok(const void *buf, uint64_t size)
{
    return (((uintptr_t)buf | size) & (DIRECT_ALIGN - 1)) == 0;
}

/* open with O_DIRECT when the buffer allows it and the filesystem takes it */
static int open_io(int dfd, const char *name, int flags, int direct, int *used)
{
    int fd = -1;

    *used = 0;
    if (direct) {
        fd = openat(dfd, name, flags | O_DIRECT | O_CLOEXEC, 0644);
        if (fd >= 0) {
            *used = 1;
            return fd;
        }
        if (errno != EINVAL)
            return -errno;
    }
    fd = openat(dfd, name, flags | O_CLOEXEC, 0644);
    return fd < 0 ? -errno : fd;
}

static int write_all(int fd, const uint8_t *buf, uint64_t size)
{
    uint64_t off = 0;

    while (off < size) {
        uint64_t chunk = size - off;
        ssize_t w;
        if (chunk > (1u << 30))
            chunk = 1u << 30;
        w = pwrite(fd, buf + off, chunk, (off_t)off);
        if (w < 0) {
            if (errno == EINTR)
                continue;
            return -errno;
        }
        if (w == 0)
            return -EIO;
        off += (uint64_t)w;
    }
    return 0;
}

static int read_all(int fd, uint8_t *buf, uint64_t size)
{
    uint64_t off = 0;

    while (off < size) {
        uint64_t chunk = size - off;
        ssize_t r;
        if (chunk > (1u << 30))
            chunk = 1u << 30;
        r = pread(fd, buf + off, chunk, (off_t)off);
        if (r < 0) {
            if (errno == EINTR)
                continue;
            return -errno;
        }
        if (r == 0)
            return -ENOENT;          /* file shorter than a record */
        off += (uint64_t)r;
    }
    return 0;
}

int disk_write(int dfd, const uint8_t *key, const void *buf, uint64_t size)
{
    char name[DISK_NAME_LEN + 1], tmp[DISK_NAME_LEN + 48];
    int fd, used, ret;

    disk_key_name(key, name);
    if (disk_stat(dfd, key, size) == 0)
        return 1;
    snprintf(tmp, sizeof(tmp), "%s.%d.%lu.tmp", name, (int)getpid(),
             (unsigned long)__atomic_fetch_add(&g_tmp_seq, 1, __ATOMIC_RELAXED));
    fd = open_io(dfd, tmp, O_CREAT | O_WRONLY | O_TRUNC, direct_ok(buf, size),
                 &used);
    if (fd < 0) {
        log_error("disk: create %s failed: %d", tmp, fd);
        return fd;
    }
    ret = write_all(fd, buf, size);
    if (ret == -EINVAL && used) {
        /* the filesystem accepted O_DIRECT at open but not the IO */
        close(fd);
        fd = open_io(dfd, tmp, O_WRONLY | O_TRUNC, 0, &used);
        ret = fd < 0 ? fd : write_all(fd, buf, size);
    }
    if (fd >= 0 && close(fd) && !ret)
        ret = -errno;
    if (!ret && renameat(dfd, tmp, dfd, name))
        ret = -errno;
    if (ret) {
        unlinkat(dfd, tmp, 0);
        log_error("disk: write %s failed: %d", name, ret);
    }
    return ret;
}

int disk_read(int dfd, const uint8_t *key, void *buf, uint64_t size)
{
    char name[DISK_NAME_LEN + 1];
    struct stat st;
    int fd, used, ret;

    disk_key_name(key, name);
    fd = open_io(dfd, name, O_RDONLY, direct_ok(buf, size), &used);
    if (fd < 0)
        return fd == -ENOENT ? -ENOENT : fd;
    if (fstat(fd, &st) || (uint64_t)st.st_size != size) {
        close(fd);
        return -ENOENT;
    }
    ret = read_all(fd, buf, size);
    if (ret == -EINVAL && used) {
        close(fd);
        fd = open_io(dfd, name, O_RDONLY, 0, &used);
        ret = fd < 0 ? fd : read_all(fd, buf, size);
    }
    if (fd >= 0)
        close(fd);
    return ret;
}
