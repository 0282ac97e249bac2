/* ref_bind_driver.c - the reference's checkpoint path, for the loader test.
 *
 * TEST INFRASTRUCTURE ONLY. Compiled with the reference's own reader
 * (src/io/dsv4_st.c) and binder (src/model/dsv4_bind.c) into
 * _ref/libdsv4ref.so by oracle/Makefile (target `ref`). It opens a directory
 * of .safetensors files, binds the model-level weights and every decoder
 * layer exactly as the reference CLI does (dsv4_bind_model, dsv4_bind_layer:
 * src/model/dsv4_bind.c:330-388), and reads every routed expert by the names
 * its expert cache resolves (src/cache/dsv4_cache.c:228-255), into the
 * structs dsv4_cuda_model_create takes. Nothing here is on the product path. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "dsv4.h"
#include "dsv4_bind.h"
#include "dsv4_st.h"

typedef struct {
    DSV4St st;
    DSV4ModelBind mb;
    DSV4LayerBind *lb;
    int nl;
    void **ebuf;          /* every expert tensor read, freed with the handle */
    size_t ne;
} RefBound;

void dsv4ref_bind_free(void *h)
{
    RefBound *b = (RefBound *)h;
    if (!b) return;
    for (size_t i = 0; i < b->ne; i++) free(b->ebuf[i]);
    free(b->ebuf);
    for (int L = 0; L < b->nl; L++) dsv4_bind_free(&b->lb[L]);
    free(b->lb);
    dsv4_bind_model_free(&b->mb);
    dsv4_st_close(&b->st);
    free(b);
}

static const void *read_named(RefBound *b, const char *name, int64_t want)
{
    const DSV4Tensor *t = dsv4_st_find(&b->st, name);
    if (!t || t->nbytes != want) {
        fprintf(stderr, "ref_bind: %s %s\n", name, t ? "has the wrong size" : "is missing");
        return NULL;
    }
    void *buf = malloc((size_t)want);
    if (!buf || dsv4_st_read(&b->st, t, buf) != want) {
        free(buf);
        return NULL;
    }
    b->ebuf[b->ne++] = buf;
    return buf;
}

/* Bind checkpoint directory `dir` for configuration c: *mw, lw[n_layers] and
 * ex[n_layers * n_experts] are filled and stay valid until the returned
 * handle is passed to dsv4ref_bind_free. NULL on any failure. */
void *dsv4ref_bind_dir(const char *dir, const DSV4Cfg *c, DSV4ModelW *mw, DSV4LayerW *lw, DSV4ExpertW *ex)
{
    RefBound *b = (RefBound *)calloc(1, sizeof *b);
    if (!b) return NULL;
    if (dsv4_st_open(&b->st, dir) != 0) { free(b); return NULL; }
    b->lb = (DSV4LayerBind *)calloc((size_t)c->n_layers, sizeof *b->lb);
    b->ebuf = (void **)calloc((size_t)c->n_layers * c->n_experts * 6, sizeof(void *));
    if (!b->lb || !b->ebuf || dsv4_bind_model(&b->st, c, 1, &b->mb) != 0) goto fail;
    *mw = b->mb.w;
    for (int L = 0; L < c->n_layers; L++) {
        if (dsv4_bind_layer(&b->st, c, L, &b->lb[L]) != 0) goto fail;
        b->nl = L + 1;
        lw[L] = b->lb[L].w;
    }
    {
        static const char *wn[3] = { "w1", "w2", "w3" };
        const int hid = c->hidden, I = c->moe_inter;
        for (int L = 0; L < c->n_layers; L++)
            for (int e = 0; e < c->n_experts; e++) {
                DSV4ExpertW *x = &ex[(size_t)L * c->n_experts + e];
                for (int i = 0; i < 3; i++) {
                    const int rows = i == 1 ? hid : I, cols = i == 1 ? I : hid;
                    char name[224];
                    snprintf(name, sizeof name, "layers.%d.ffn.experts.%d.%s.weight", L, e, wn[i]);
                    const void *w = read_named(b, name, (int64_t)rows * (cols / 2));
                    snprintf(name, sizeof name, "layers.%d.ffn.experts.%d.%s.scale", L, e, wn[i]);
                    const void *s = read_named(b, name, (int64_t)rows * (cols / 32));
                    if (!w || !s) goto fail;
                    DSV4QMat q = { w, s, DSV4_WFP4, rows, cols, 1, 32 };
                    if (i == 0) x->w1 = q;
                    else if (i == 1) x->w2 = q;
                    else x->w3 = q;
                }
            }
    }
    return b;
fail:
    dsv4ref_bind_free(b);
    return NULL;
}
