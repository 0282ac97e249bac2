/* Prints sizeof/offsetof of the model-level structs. Compiled twice by
 * tests/golden/make_layout.py: once against the reference's dsv4.h (golden,
 * where the reference checkout exists) and once against include/dsv4_types.h
 * (tests/test_layout_cpu.py); the two outputs must agree. */
#include <stdio.h>
#include <stddef.h>
#ifdef USE_REF
#include "dsv4.h"
#else
#include "dsv4_types.h"
#endif
#define S(T) printf("sizeof %s %zu\n", #T, sizeof(T))
#define O(T, f) printf("offsetof %s.%s %zu\n", #T, #f, offsetof(T, f))
int main(void)
{
    S(DSV4Cfg); S(DSV4QMat); S(DSV4CompressorW); S(DSV4IndexerW); S(DSV4AttnW);
    S(DSV4ExpertW); S(DSV4MoeW); S(DSV4HcW); S(DSV4LayerW); S(DSV4ModelW);
    O(DSV4Cfg, hidden); O(DSV4Cfg, max_pos); O(DSV4Cfg, sliding_window); O(DSV4Cfg, index_topk);
    O(DSV4Cfg, compress_ratios); O(DSV4Cfg, compress_rope_theta); O(DSV4Cfg, hc_eps);
    O(DSV4Cfg, moe_inter); O(DSV4Cfg, routed_scale); O(DSV4Cfg, topk_method); O(DSV4Cfg, swiglu_limit);
    O(DSV4Cfg, yarn_orig_ctx); O(DSV4Cfg, wblock_n); O(DSV4Cfg, num_nextn_predict);
    O(DSV4QMat, wdt); O(DSV4QMat, blk_c);
    O(DSV4CompressorW, wkv); O(DSV4CompressorW, wgate); O(DSV4CompressorW, ratio); O(DSV4CompressorW, coff);
    O(DSV4IndexerW, weights_proj); O(DSV4IndexerW, comp);
    O(DSV4AttnW, wq_a); O(DSV4AttnW, wo_b); O(DSV4AttnW, comp); O(DSV4AttnW, idx); O(DSV4AttnW, has_idx);
    O(DSV4MoeW, bias); O(DSV4MoeW, tid2eid); O(DSV4MoeW, shared);
    O(DSV4LayerW, attn); O(DSV4LayerW, moe); O(DSV4LayerW, hc_attn); O(DSV4LayerW, hc_ffn);
    O(DSV4LayerW, layer); O(DSV4LayerW, has_idx);
    O(DSV4ModelW, norm); O(DSV4ModelW, hc_head); O(DSV4ModelW, wdt);
    return 0;
}
