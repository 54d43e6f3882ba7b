// vkllm_tensor over CUDA memory (reference: src/core/vkllm_tensor.c).
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "internal.h"

namespace
{

// Contiguous byte strides, W innermost (reference: src/core/vkllm_tensor.c:13-31).
vkllm_err_t calc_strides(const uint32_t *shapes, vkllm_dtype_t dtype, uint32_t *strides)
{
    struct vkllm_dtype_info info;
    _CHECK(vkllm_get_dtype_info(dtype, &info));
    uint64_t row = (uint64_t)shapes[3] * info.bytes;
    uint64_t s1 = (uint64_t)shapes[2] * row;
    uint64_t s0 = (uint64_t)shapes[1] * s1;
    if (s0 > 0xffffffffull || s0 * shapes[0] > 0xffffffffull)
    {
        log_error("tensor of %u x %u x %u x %u elements exceeds the 4 GiB byte-stride range", shapes[0], shapes[1],
                  shapes[2], shapes[3]);
        return VKLLM_ERR_ARGS;
    }
    strides[3] = info.bytes;
    strides[2] = (uint32_t)row;
    strides[1] = (uint32_t)s1;
    strides[0] = (uint32_t)s0;
    return VKLLM_ERR_OK;
}

// name = a + b, a cut so that the whole fits (what "%.{127 - |b|}s%s" prints), without printf: views
// are created per token by the graph builders.
void set_name(vkllm_tensor *t, const char *a, const char *b)
{
    char *n = (char *)t->name;
    const size_t lb = strnlen(b, sizeof(t->name) - 1), la = strnlen(a, sizeof(t->name) - 1 - lb);
    memcpy(n, a, la);
    memcpy(n + la, b, lb);
    n[la + lb] = 0;
}

// Tensor structs come from a per-context free list when their params block fits kPoolParams bytes:
// the graph builders create and free ~20 nodes per layer every token. A 16-byte header before the
// struct records whether the block has the pooled size.
constexpr size_t kPoolParams = 64, kTensorHdr = 16;

vkllm_tensor *tensor_alloc(vkllm_context *ctx, size_t params_bytes)
{
    const bool pooled = ctx && ctx->runtime && params_bytes <= kPoolParams;
    const size_t bytes = kTensorHdr + sizeof(vkllm_tensor) + (pooled ? kPoolParams : params_bytes);
    unsigned char *b = nullptr;
    if (pooled && !ctx->runtime->tensor_pool.empty())
    {
        b = (unsigned char *)ctx->runtime->tensor_pool.back();
        ctx->runtime->tensor_pool.pop_back();
        memset(b, 0, bytes);
    }
    else
        b = (unsigned char *)calloc(1, bytes);
    if (!b)
        return nullptr;
    b[0] = pooled ? 1 : 0;
    return (vkllm_tensor *)(b + kTensorHdr);
}

void tensor_release(vkllm_context *ctx, vkllm_tensor *t)
{
    unsigned char *b = (unsigned char *)t - kTensorHdr;
    if (b[0] && ctx && ctx->runtime && ctx->runtime->tensor_pool.size() < 4096)
        ctx->runtime->tensor_pool.push_back(b);
    else
        free(b);
}

} // namespace

namespace vkb
{

vkllm_tensor *storage_owner(vkllm_tensor *t)
{
    int guard = 0;
    while (t && t->data.is_ref && t->srcs[0] && guard++ < 64)
        t = t->srcs[0];
    return t;
}

void *dev_ptr(vkllm_context *ctx, vkllm_tensor *t)
{
    vkllm_tensor *o = storage_owner(t);
    if (!o)
        return nullptr;
    if (!o->data.dev)
    {
        size_t cap = 0;
        void *p = ctx->runtime->dev_alloc->alloc(o->bytes, &cap);
        if (!p)
        {
            log_error("device allocation of %u bytes for tensor %s failed", o->bytes, o->name);
            return nullptr;
        }
        o->data.dev = p;
        o->data.capacity = cap;
    }
    if (t != o)
        t->data.dev = o->data.dev;
    return o->data.dev;
}

Strides4 elem_strides(const vkllm_tensor *t)
{
    Strides4 r;
    uint32_t b = dtype_bytes(t->dtype);
    for (int i = 0; i < 4; ++i)
        r.s[i] = b ? t->strides[i] / b : 0;
    return r;
}

} // namespace vkb

extern "C" vkllm_err_t vkllm_tensor_new(struct vkllm_context *context, const char *name, const uint32_t *shapes,
                                        vkllm_dtype_t dtype, vkllm_op_t op, struct vkllm_tensor **srcs,
                                        const uint32_t n_srcs, const void *params, size_t params_bytes, bool mapped,
                                        struct vkllm_tensor **p)
{
    _CHECK_ARGS(context && p);
    if (!shapes)
    {
        log_error("shape is empty. shapes is NULL");
        return VKLLM_ERR_ARGS;
    }
    for (uint32_t i = 0; i < 4; ++i)
    {
        if (shapes[i] == 0)
        {
            log_error("shape is empty. shapes[%u] is 0", i);
            return VKLLM_ERR_ARGS;
        }
    }
    _CHECK_ARGS(n_srcs <= VKLLM_MAX_SRCS);
    _CHECK_ARGS(n_srcs == 0 || srcs);

    vkllm_tensor *t = tensor_alloc(context, params_bytes);
    if (!t)
        return VKLLM_ERR_ALLOC;
    if (name)
    {
        const size_t ln = strnlen(name, sizeof(t->name) - 1);
        memcpy((char *)t->name, name, ln); // calloc'd: the terminator is already there
    }
    t->dtype = dtype;
    memcpy(t->shapes, shapes, sizeof(t->shapes));
    vkllm_err_t err = calc_strides(shapes, dtype, t->strides);
    if (err != VKLLM_ERR_OK)
    {
        tensor_release(context, t);
        return err;
    }
    uint64_t total = (uint64_t)shapes[0] * t->strides[0];
    t->bytes = (uint32_t)((total + 63) / 64 * 64);
    t->device = context->device;
    t->op = op;
    for (uint32_t i = 0; i < n_srcs; ++i)
        t->srcs[i] = srcs[i];
    if (params && params_bytes)
        memcpy(t->params, params, params_bytes);
    t->data.mapped = mapped;
    t->data.is_ref = false;
    if (mapped)
    {
        size_t cap = 0;
        void *h = context->runtime->host_alloc->alloc(t->bytes, &cap);
        if (!h)
        {
            log_error("pinned host allocation of %u bytes failed", t->bytes);
            tensor_release(context, t);
            return VKLLM_ERR_ALLOC;
        }
        void *d = nullptr;
        if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess)
        {
            (void)cudaGetLastError();
            context->runtime->host_alloc->release(h);
            tensor_release(context, t);
            return VKLLM_ERR_VULKAN;
        }
        // Fresh mapped memory reads as zero in the reference (a new host-visible allocation); this
        // buffer may be recycled from the pinned-host cache, so clear it.
        memset(h, 0, t->bytes);
        t->data.host = h;
        t->data.dev = d;
        t->data.capacity = cap;
    }
    t->pipeline = NULL;
    context->stats.tensor_alloc_counts += 1;
    *p = t;
    return VKLLM_ERR_OK;
}

extern "C" void vkllm_tensor_free(struct vkllm_context *context, struct vkllm_tensor *tensor)
{
    if (!tensor)
        return;
    if (!tensor->data.is_ref && context)
    {
        if (tensor->data.mapped)
            context->runtime->host_alloc->release(tensor->data.host);
        else if (tensor->data.dev)
            context->runtime->dev_alloc->release(tensor->data.dev);
    }
    tensor_release(context, tensor);
    if (context)
        context->stats.tensor_free_counts += 1;
}

extern "C" vkllm_err_t vkllm_tensor_flush_cache(struct vkllm_context *context, struct vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && tensor);
    if (!tensor->data.mapped)
    {
        log_error("can only flush mapped buffer.");
        return VKLLM_ERR_ARGS;
    }
    // Pinned mapped memory is coherent; a full fence orders the host writes before later launches.
    __sync_synchronize();
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_tensor_invalid_cache(struct vkllm_context *context, struct vkllm_tensor *tensor)
{
    _CHECK_ARGS(context && tensor);
    if (!tensor->data.mapped)
    {
        log_error("can only invalid mapped buffer.");
        return VKLLM_ERR_ARGS;
    }
    __sync_synchronize();
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_tensor_new_staging(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                                struct vkllm_tensor **staging)
{
    _CHECK_ARGS(context && tensor && staging);
    _CHECK(vkllm_tensor_new(context, "", tensor->shapes, tensor->dtype, tensor->op, tensor->srcs, 4, NULL, 0, true,
                            staging));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_tensor_reshape(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                            const uint32_t *shapes)
{
    _CHECK_ARGS(context && tensor && shapes);
    _CHECK_ARGS((uint64_t)_MUL4(tensor->shapes) == (uint64_t)_MUL4(shapes));
    for (int i = 0; i < 4; ++i)
        _CHECK_ARGS(shapes[i] > 0);
    memcpy(tensor->shapes, shapes, sizeof(tensor->shapes));
    _CHECK(calc_strides(shapes, tensor->dtype, tensor->strides));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_tensor_permute(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                            const uint32_t *axis)
{
    _CHECK_ARGS(context && tensor && axis);
    uint32_t seen = 0;
    for (int i = 0; i < 4; ++i)
    {
        _CHECK_ARGS(axis[i] < 4);
        seen |= 1u << axis[i];
    }
    _CHECK_ARGS(seen == 0xfu);
    uint32_t shapes[4], strides[4];
    memcpy(shapes, tensor->shapes, sizeof(shapes));
    memcpy(strides, tensor->strides, sizeof(strides));
    for (int i = 0; i < 4; ++i)
    {
        tensor->shapes[i] = shapes[axis[i]];
        tensor->strides[i] = strides[axis[i]];
    }
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_tensor_copy_ref(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                             struct vkllm_tensor **p)
{
    _CHECK_ARGS(context && tensor && p);
    vkllm_tensor *t = tensor_alloc(context, 0);
    if (!t)
        return VKLLM_ERR_ALLOC;
    set_name(t, tensor->name, "_ref");
    t->dtype = tensor->dtype;
    memcpy(t->shapes, tensor->shapes, sizeof(t->shapes));
    memcpy(t->strides, tensor->strides, sizeof(t->strides));
    t->bytes = tensor->bytes;
    t->device = tensor->device;
    t->data.dev = tensor->data.dev;
    t->data.host = tensor->data.host;
    t->data.mapped = tensor->data.mapped;
    t->data.capacity = tensor->data.capacity;
    t->data.is_ref = true;
    t->op = VKLLM_OP_REF;
    t->pipeline = NULL;
    t->srcs[0] = tensor;
    context->stats.tensor_alloc_counts += 1;
    *p = t;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_tensor_slice0(struct vkllm_context *context, struct vkllm_tensor *tensor,
                                           uint32_t extents[4], struct vkllm_tensor **slice)
{
    _CHECK_ARGS(context && tensor && extents && slice);
    for (int i = 0; i < 4; ++i)
        _CHECK_ARGS(extents[i] > 0 && extents[i] <= tensor->shapes[i]);
    _CHECK(vkllm_tensor_copy_ref(context, tensor, slice));
    vkllm_tensor *t = *slice;
    set_name(t, tensor->name, "_slice0");
    memcpy(t->shapes, extents, sizeof(t->shapes));
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_tensor_s(struct vkllm_context *context, struct vkllm_tensor *tensor, char *buf,
                                      size_t len)
{
    _CHECK_ARGS(context && tensor && buf && len > 0);
    int n = snprintf(buf, len, "%s<%s>[%u, %u, %u, %u]", tensor->name, vkllm_dtype_s(tensor->dtype),
                     tensor->shapes[0], tensor->shapes[1], tensor->shapes[2], tensor->shapes[3]);
    if (n < 0 || (size_t)n >= len)
        return VKLLM_ERR_ARGS;
    return VKLLM_ERR_OK;
}
