/*
 * Disk tier: one file per record, named by the 64 lowercase hex digits of
 * its 32-byte key (CrossCache src/cache/cache.c:222-278, CACHEKEY_TO_NAME,
 * lookup_file, write_to_file, read_from_file).
 *
 * Differences, by design:
 *   - files live in one subdirectory per (model tag, tp size, tp rank)
 *     under the root, "<tag>.tp<size>.<rank>" with '/' and non-printable
 *     characters of the tag replaced by '_'.  The reference puts every
 *     record of every model and rank in the root directory, so two tensor-
 *     parallel ranks (different head shards, same key) or two models that
 *     saw the same prompt overwrite each other's files;
 *   - a record is written to a temporary name and renamed into place, so a
 *     reader never sees a partial file; a file counts as present only when
 *     its size equals the record size;
 *   - short reads and writes are retried to completion and reported
 *     (the reference logs them and returns success).
 * Records are written with O_DIRECT (the pool is page aligned and records
 * are multiples of 4 KiB); filesystems that refuse O_DIRECT get buffered IO.
 */
#ifndef CC_DISK_H
#define CC_DISK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DISK_NAME_LEN 64

/* open (creating one level if missing) the root directory: fd or -errno */
int disk_open_root(const char *root);

/* open (creating if missing) the namespace directory of one runtime entry
 * below the root: fd or -errno */
int disk_open_ns(int rootfd, const char *tag, uint8_t tp_size, uint8_t tp_id);

/* 64 hex digits + NUL */
void disk_key_name(const uint8_t *key, char name[DISK_NAME_LEN + 1]);

/* 0 when the record file of `key` exists with exactly `size` bytes,
 * -ENOENT otherwise */
int disk_stat(int dfd, const uint8_t *key, uint64_t size);

/* write `size` bytes as the record of `key`: 0 written, 1 already present
 * with the right size (nothing written), -errno on failure */
int disk_write(int dfd, const uint8_t *key, const void *buf, uint64_t size);

/* read the record of `key` into buf: 0, -ENOENT (missing or wrong size) or
 * -errno */
int disk_read(int dfd, const uint8_t *key, void *buf, uint64_t size);

#ifdef __cplusplus
}
#endif

#endif
