/* Bounded safetensors reader for the B200 backend's host side.
 *
 * Admission matches the reference reader (src/safetensors.c:367-427): an
 * 8-byte little-endian header length in [2, 1 MiB] that fits the file; a JSON
 * object whose first byte is '{'; tensor entries holding exactly dtype, shape
 * and data_offsets; dtypes F8_E4M3, BF16, F32, I64; rank <= 8; unique printable
 * ASCII names (JSON escapes allowed); at most one "__metadata__" object of
 * string values; byte ranges that match their element counts and tile the data
 * region with no gap, overlap or trailing bytes. Reads use pread and never
 * share a file position, so concurrent reads of one handle are safe.
 */
#ifndef LUN_ST_H
#define LUN_ST_H

#include <stddef.h>
#include <stdint.h>

#define LUN_ST_MAX_NAME 256
#define LUN_ST_MAX_DIMS 8
#define LUN_ST_MAX_TENSORS 4096
#define LUN_ST_MAX_HEADER (1024u * 1024u)

/* Enumerator value is the element size in bytes. */
typedef enum {
    LUN_F8_E4M3 = 1,
    LUN_BF16 = 2,
    LUN_F32 = 4,
    LUN_I64 = 8
} lun_dtype;

typedef struct {
    char name[LUN_ST_MAX_NAME];
    lun_dtype dtype;
    size_t rank;
    uint64_t shape[LUN_ST_MAX_DIMS];
    uint64_t begin, end; /* relative to the data region */
} lun_tensor;

typedef struct {
    int fd;
    uint64_t file_bytes;
    uint64_t data_base; /* 8 + header length */
    size_t count;
    lun_tensor *tensors;
} lun_st;

int lun_st_open(lun_st *s, const char *path, char *error, size_t capacity);
void lun_st_close(lun_st *s);
const lun_tensor *lun_st_find(const lun_st *s, const char *name);
/* Exact bounded read of [offset, offset+bytes) of tensor t (which must belong to s). */
int lun_st_read(const lun_st *s, const lun_tensor *t, uint64_t offset, void *out, size_t bytes);

float lun_bf16_to_f32(uint16_t bits);
/* E4M3FN code -> FP32, exact; both NaN codes (0x7f, 0xff) give NaN. */
float lun_e4m3_to_f32(unsigned char code);

#endif
