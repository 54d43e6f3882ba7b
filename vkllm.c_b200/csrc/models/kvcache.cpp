// Per-layer fp16 KV cache (reference: src/models/vkllm_kvcache.c).
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../runtime/internal.h"
#include "vkllm_kvcache.h"

extern "C" vkllm_err_t vkllm_kvcache_new(struct vkllm_context *context, uint32_t kcache_shape[4],
                                         uint32_t vcache_shape[4], uint32_t layer_counts,
                                         struct vkllm_kvcache **kvcache)
{
    _CHECK_ARGS(context && kcache_shape && vcache_shape && kvcache);
    vkllm_kvcache *p = (vkllm_kvcache *)calloc(1, sizeof(vkllm_kvcache));
    if (!p)
        return VKLLM_ERR_ALLOC;
    p->layer_counts = layer_counts;
    memcpy(p->kcache_shape, kcache_shape, sizeof(p->kcache_shape));
    memcpy(p->vcache_shape, vcache_shape, sizeof(p->vcache_shape));
    vkllm_err_t err = vkllm_array_tensor_new(&p->kcaches, layer_counts);
    if (err == VKLLM_ERR_OK)
        err = vkllm_array_tensor_new(&p->vcaches, layer_counts);
    char name[128];
    uint32_t offsets = 0;
    for (uint32_t i = 0; err == VKLLM_ERR_OK && i < layer_counts; ++i)
    {
        vkllm_tensor *k = nullptr, *v = nullptr;
        snprintf(name, sizeof(name), "kcache_%u", i);
        err = vkllm_tensor_new(context, name, kcache_shape, vkllm_dtype_float16, VKLLM_OP_UPDATE_ROWS, NULL, 0,
                               &offsets, sizeof(offsets), false, &k);
        if (err != VKLLM_ERR_OK)
            break;
        vkllm_array_tensor_append(p->kcaches, k);
        snprintf(name, sizeof(name), "vcache_%u", i);
        err = vkllm_tensor_new(context, name, vcache_shape, vkllm_dtype_float16, VKLLM_OP_UPDATE_ROWS, NULL, 0,
                               &offsets, sizeof(offsets), false, &v);
        if (err != VKLLM_ERR_OK)
            break;
        vkllm_array_tensor_append(p->vcaches, v);
        // The cache is persistent: back it now and zero it, so unwritten rows read as 0.
        void *kd = vkb::dev_ptr(context, k), *vd = vkb::dev_ptr(context, v);
        if (!kd || !vd)
        {
            err = VKLLM_ERR_ALLOC;
            break;
        }
        if (cudaMemsetAsync(kd, 0, k->bytes, context->runtime->stream) != cudaSuccess ||
            cudaMemsetAsync(vd, 0, v->bytes, context->runtime->stream) != cudaSuccess)
        {
            err = VKLLM_ERR_VULKAN;
            break;
        }
    }
    if (err != VKLLM_ERR_OK)
    {
        vkllm_kvcache_free(context, p);
        return err;
    }
    cudaStreamSynchronize(context->runtime->stream);
    *kvcache = p;
    return VKLLM_ERR_OK;
}

extern "C" vkllm_err_t vkllm_kvcache_update(struct vkllm_context *context, struct vkllm_kvcache *kvcache,
                                            struct vkllm_tensor **key, struct vkllm_tensor **value, uint32_t layer,
                                            uint32_t offset)
{
    _CHECK_ARGS(context && kvcache && key && value);
    vkllm_tensor *pkey = *key, *pvalue = *value;
    _CHECK_ARGS(pkey && pvalue);
    _CHECK_ARGS(layer < kvcache->kcaches->used_n && layer < kvcache->vcaches->used_n);
    vkllm_tensor *kc = kvcache->kcaches->data[layer];
    vkllm_tensor *vc = kvcache->vcaches->data[layer];
    _CHECK_ARGS(pkey->shapes[0] <= kc->shapes[0] && pkey->shapes[1] <= kc->shapes[1]);
    _CHECK_ARGS((uint64_t)pkey->shapes[2] + offset <= kc->shapes[2] && pkey->shapes[3] <= kc->shapes[3]);
    _CHECK_ARGS(pvalue->shapes[0] <= vc->shapes[0] && pvalue->shapes[1] <= vc->shapes[1]);
    _CHECK_ARGS((uint64_t)pvalue->shapes[2] + offset <= vc->shapes[2] && pvalue->shapes[3] <= vc->shapes[3]);

    kc->srcs[0] = pkey;
    memcpy(kc->params, &offset, sizeof(offset));
    vc->srcs[0] = pvalue;
    memcpy(vc->params, &offset, sizeof(offset));
    kc->pipeline = NULL; // re-selected for the new source
    vc->pipeline = NULL;

    uint32_t extents[4] = {pkey->shapes[0], pkey->shapes[1], pkey->shapes[2] + offset, pkey->shapes[3]};
    _CHECK(vkllm_tensor_slice0(context, kc, extents, key));
    uint32_t vext[4] = {pvalue->shapes[0], pvalue->shapes[1], pvalue->shapes[2] + offset, pvalue->shapes[3]};
    _CHECK(vkllm_tensor_slice0(context, vc, vext, value));
    return VKLLM_ERR_OK;
}

extern "C" void vkllm_kvcache_free(struct vkllm_context *context, struct vkllm_kvcache *kvcache)
{
    if (!kvcache)
        return;
    if (kvcache->vcaches)
    {
        for (size_t i = 0; i < kvcache->vcaches->used_n; ++i)
            vkllm_tensor_free(context, kvcache->vcaches->data[i]);
        vkllm_array_tensor_free(kvcache->vcaches);
    }
    if (kvcache->kcaches)
    {
        for (size_t i = 0; i < kvcache->kcaches->used_n; ++i)
            vkllm_tensor_free(context, kvcache->kcaches->data[i]);
        vkllm_array_tensor_free(kvcache->kcaches);
    }
    free(kvcache);
}
