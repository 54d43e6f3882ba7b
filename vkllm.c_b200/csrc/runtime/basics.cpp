// Error/dtype/op names, the logger and the timing hashmap of the public C API.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "vkllm_dtypes.h"
#include "vkllm_errors.h"
#include "vkllm_hashmap.h"
#include "vkllm_log.h"
#include "vkllm_ops.h"

extern "C" const char *vkllm_err_s(vkllm_err_t err)
{
    // Indexed by err - 1 like the reference (src/core/vkllm_errors.c:3-13).
    static const char *const names[] = {"VKLLM_ERR_OK",          "VKLLM_ERR_ALLOC",
                                        "VKLLM_ERR_VULKAN",      "VKLLM_ERR_DEV_NOT_FOUND",
                                        "VKLLM_ERR_PIPELINE_NOT_FOUND", "VKLLM_ERR_ARGS"};
    int i = (int)err - 1;
    if (i < 0 || i >= (int)(sizeof(names) / sizeof(names[0])))
        return "VKLLM_ERR_UNKNOWN";
    return names[i];
}

extern "C" const char *vkllm_dtype_s(vkllm_dtype_t dtype)
{
    static const char *const names[] = {"vkllm_dtype_start", "float32", "float16", "int8", "uint32"};
    int i = (int)dtype;
    if (i < 0 || i >= (int)(sizeof(names) / sizeof(names[0])))
        return "unknown";
    return names[i];
}

extern "C" vkllm_err_t vkllm_get_dtype_info(vkllm_dtype_t dtype, struct vkllm_dtype_info *info)
{
    if (!info)
        return VKLLM_ERR_ARGS;
    uint32_t bytes = 0;
    switch (dtype)
    {
    case vkllm_dtype_float32:
    case vkllm_dtype_uint32:
        bytes = 4;
        break;
    case vkllm_dtype_float16:
        bytes = 2;
        break;
    case vkllm_dtype_int8:
        bytes = 1;
        break;
    default:
        log_error("%s dtype is unsupported", vkllm_dtype_s(dtype));
        return VKLLM_ERR_ARGS;
    }
    info->dtype = dtype;
    info->bytes = bytes;
    info->items_per_block = 1;
    info->bytes_per_block = bytes;
    return VKLLM_ERR_OK;
}

extern "C" const char *vkllm_op_s(const vkllm_op_t op)
{
    static const char *const names[] = {"VKLLM_OP_NONE",    "VKLLM_OP_COPY",        "VKLLM_OP_BIN",
                                        "VKLLM_OP_EMBEDDING", "VKLLM_OP_RMSNORM",   "VKLLM_OP_MATMUL",
                                        "VKLLM_OP_ROPE",    "VKLLM_OP_SOFTMAX",     "VKLLM_OP_FFN_UP_AND_GATE",
                                        "VKLLM_OP_UPDATE_ROWS", "VKLLM_OP_ARG_MAX", "VKLLM_OP_REF"};
    int i = (int)op;
    if (i < 0 || i >= (int)(sizeof(names) / sizeof(names[0])))
        return "VKLLM_OP_UNKNOWN";
    return names[i];
}

// ---------------------------------------------------------------------------------------------
// Logger
static int g_log_level = -1;

extern "C" void vkllm_log_set_level(int level)
{
    g_log_level = level;
}

extern "C" void vkllm_log(int level, const char *file, int line, const char *fmt, ...)
{
    if (g_log_level < 0)
    {
        const char *e = getenv("VKLLM_LOG_LEVEL");
        g_log_level = e ? atoi(e) : VKLLM_LOG_WARN;
    }
    if (level < g_log_level)
        return;
    static const char *const lv[] = {"TRACE", "DEBUG", "INFO", "WARN", "ERROR", "FATAL"};
    const char *base = strrchr(file, '/');
    fprintf(stderr, "[vkllm %s] %s:%d: ", lv[level < 0 ? 0 : (level > 5 ? 5 : level)], base ? base + 1 : file, line);
    va_list ap;
    va_start(ap, fmt);
    vfprintf(stderr, fmt, ap);
    va_end(ap);
    fputc('\n', stderr);
}

// ---------------------------------------------------------------------------------------------
// Hashmap (string -> uint64), open addressing with linear probing and tombstones.
static const char *const kTombstone = "\x01tombstone";

extern "C" uint64_t vkllm_hashmap_hash(const char *key, size_t capacity)
{
    uint64_t h = 1469598103934665603ull; // FNV-1a
    for (const unsigned char *p = (const unsigned char *)key; *p; ++p)
        h = (h ^ *p) * 1099511628211ull;
    return capacity ? h % capacity : h;
}

extern "C" vkllm_err_t vkllm_hashmap_new(struct vkllm_hashmap **map, size_t init_capacity)
{
    if (!map)
        return VKLLM_ERR_ARGS;
    struct vkllm_hashmap *m = (struct vkllm_hashmap *)calloc(1, sizeof(*m));
    if (!m)
        return VKLLM_ERR_ALLOC;
    m->capacity = init_capacity < 8 ? 8 : init_capacity;
    m->entries = (struct vkllm_hashmap_entry *)calloc(m->capacity, sizeof(struct vkllm_hashmap_entry));
    if (!m->entries)
    {
        free(m);
        return VKLLM_ERR_ALLOC;
    }
    *map = m;
    return VKLLM_ERR_OK;
}

static void free_key(struct vkllm_hashmap_entry *e)
{
    if (e->key && e->key != kTombstone)
        free(e->key);
    e->key = NULL;
}

extern "C" void vkllm_hashmap_free(struct vkllm_hashmap *map)
{
    if (!map)
        return;
    for (size_t i = 0; i < map->capacity; ++i)
        free_key(&map->entries[i]);
    free(map->entries);
    free(map);
}

static long find_slot(const struct vkllm_hashmap *m, const char *key)
{
    size_t i = (size_t)vkllm_hashmap_hash(key, m->capacity);
    for (size_t n = 0; n < m->capacity; ++n, i = (i + 1) % m->capacity)
    {
        const struct vkllm_hashmap_entry *e = &m->entries[i];
        if (!e->occupied && e->key != kTombstone)
            return -1;
        if (e->occupied && strcmp(e->key, key) == 0)
            return (long)i;
    }
    return -1;
}

extern "C" vkllm_err_t vkllm_hashmap_resize(struct vkllm_hashmap *map, size_t new_capacity)
{
    if (!map || new_capacity < map->size + 1)
        return VKLLM_ERR_ARGS;
    struct vkllm_hashmap_entry *old = map->entries;
    size_t old_cap = map->capacity;
    map->entries = (struct vkllm_hashmap_entry *)calloc(new_capacity, sizeof(struct vkllm_hashmap_entry));
    if (!map->entries)
    {
        map->entries = old;
        return VKLLM_ERR_ALLOC;
    }
    map->capacity = new_capacity;
    map->size = 0;
    map->tombstones = 0;
    for (size_t i = 0; i < old_cap; ++i)
    {
        if (old[i].occupied)
        {
            size_t j = (size_t)vkllm_hashmap_hash(old[i].key, new_capacity);
            while (map->entries[j].occupied)
                j = (j + 1) % new_capacity;
            map->entries[j] = old[i];
            map->size++;
        }
    }
    free(old);
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_hashmap_insert(struct vkllm_hashmap *map, const char *key, uint64_t value)
{
    if (!map || !key)
        return VKLLM_ERR_ARGS;
    long s = find_slot(map, key);
    if (s >= 0)
    {
        map->entries[s].value = value;
        return VKLLM_ERR_OK;
    }
    if ((map->size + map->tombstones + 1) * 4 > map->capacity * 3)
    {
        vkllm_err_t e = vkllm_hashmap_resize(map, map->capacity * 2);
        if (e != VKLLM_ERR_OK)
            return e;
    }
    size_t i = (size_t)vkllm_hashmap_hash(key, map->capacity);
    while (map->entries[i].occupied)
        i = (i + 1) % map->capacity;
    struct vkllm_hashmap_entry *e = &map->entries[i];
    if (e->key == kTombstone)
        map->tombstones--;
    e->key = strdup(key);
    if (!e->key)
        return VKLLM_ERR_ALLOC;
    e->value = value;
    e->occupied = true;
    map->size++;
    return VKLLM_ERR_OK;
}

extern "C" bool vkllm_hashmap_get(const struct vkllm_hashmap *map, const char *key, uint64_t *out_value)
{
    if (!map || !key)
        return false;
    long s = find_slot(map, key);
    if (s < 0)
        return false;
    if (out_value)
        *out_value = map->entries[s].value;
    return true;
}

extern "C" bool vkllm_hashmap_contains(const struct vkllm_hashmap *map, const char *key)
{
    return vkllm_hashmap_get(map, key, NULL);
}

extern "C" vkllm_err_t vkllm_hashmap_remove(struct vkllm_hashmap *map, const char *key)
{
    if (!map || !key)
        return VKLLM_ERR_ARGS;
    long s = find_slot(map, key);
    if (s < 0)
        return VKLLM_ERR_OK; // removing an absent key is not an error (src/core/vkllm_hashmap.c:197-215)
    free_key(&map->entries[s]);
    map->entries[s].key = (char *)kTombstone;
    map->entries[s].occupied = false;
    map->size--;
    map->tombstones++;
    return VKLLM_ERR_OK;
}

extern "C" void vkllm_hashmap_clear(struct vkllm_hashmap *map)
{
    if (!map)
        return;
    for (size_t i = 0; i < map->capacity; ++i)
    {
        free_key(&map->entries[i]);
        map->entries[i].occupied = false;
        map->entries[i].value = 0;
    }
    map->size = 0;
    map->tombstones = 0;
}

extern "C" size_t vkllm_hashmap_size(const struct vkllm_hashmap *map)
{
    return map ? map->size : 0;
}

extern "C" bool vkllm_hashmap_empty(const struct vkllm_hashmap *map)
{
    return vkllm_hashmap_size(map) == 0;
}
