/* trunk_ref.c - test infrastructure only: flat accessors around the
 * REFERENCE's own trunk manifest reader (src/50_loader/dsv4_trunk_manifest.c
 * dsv4_trunk_load_manifest), so the CPU tests can check the
 * library's trunk.idx reader against it record by record. Compiled by
 * oracle/Makefile into _ref/libdsv4trunk.so with the reference's sources read
 * where they lie; nothing here is called by the library. */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "dsv4_trunk.h"

/* The record layout the tests read (the library's dsv4cu_trunk_tensor). */
typedef struct {
    int32_t slot, dtype, rows, cols, wdt, blk_r, blk_c;
    int64_t off, nbytes;
} RefTrunkTensor;

static void ref_trunk_release(DSV4Trunk *tr)
{
    if (tr->lay)
        for (int L = 0; L < tr->n_layers; L++) free(tr->lay[L].t);
    free(tr->lay);
}

/* 0 and n_layers for a manifest the reference accepts, -1 when it rejects it.
 * For layer >= 0 also run[0..2] (file offset, bytes, widen bytes), the tensor
 * count and up to cap records in manifest order. */
int ref_trunk_manifest(const char *dir, int *n_layers, int layer, int64_t *run, int *n_tensors,
                       RefTrunkTensor *out, int cap)
{
    DSV4Trunk tr;
    memset(&tr, 0, sizeof tr);
    tr.fd = -1;
    tr.bfd = -1;
    const int rc = dsv4_trunk_load_manifest(&tr, dir);
    if (rc != 0) {
        ref_trunk_release(&tr);
        return -1;
    }
    if (n_layers) *n_layers = tr.n_layers;
    if (layer >= 0 && layer < tr.n_layers) {
        const DSV4TrunkLayer *lay = &tr.lay[layer];
        if (run) {
            run[0] = lay->file_off;
            run[1] = lay->nbytes;
            run[2] = lay->widen_bytes;
        }
        if (n_tensors) *n_tensors = lay->nt;
        for (int i = 0; out && i < cap && i < lay->nt; i++) {
            const DSV4TrunkTensor *t = &lay->t[i];
            out[i].slot = t->slot;
            out[i].dtype = t->dtype;
            out[i].rows = t->rows;
            out[i].cols = t->cols;
            out[i].wdt = t->wdt;
            out[i].blk_r = t->blk_r;
            out[i].blk_c = t->blk_c;
            out[i].off = t->off;
            out[i].nbytes = t->nbytes;
        }
    }
    ref_trunk_release(&tr);
    return 0;
}
