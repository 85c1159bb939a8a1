/* ref_flash_wrap.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Builds the reference's flash.c, unmodified and read where it lies (REF_DIR on the include
 * path), into oracle/_ref/libflashref.so, with oracle/sve_shim standing in for arm_sve.h.
 * flash.c keeps attn_flash / attn_ref static inside its single translation unit, so this
 * file includes that unit and exports thin forwarders. Its main() is renamed and exported
 * too, so the reference's own CLI suite can be run from the library.
 */
#define main flash_ref_main
#include <flash.c>
#undef main

void ref_attn_flash(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq, int Hkv, int Sq,
                    int Sk, int D, int causal, int bk, void *scratch, int v_prepacked) {
    attn_flash(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, bk, scratch, v_prepacked, NULL);
}

void ref_attn_ref(const uint16_t *Q, const uint16_t *K, const uint16_t *V, float *O, int Hq, int Hkv, int Sq,
                  int Sk, int D, int causal, const int *rows, int nrows) {
    attn_ref(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, rows, nrows);
}

size_t ref_scratch_bytes(int D, int bk) { return attn_flash_scratch_bytes(D, bk); }

void ref_pack_v_full(const uint16_t *V, uint16_t *Vp, int Hkv, int Sk, int D) { pack_v_full(V, Vp, Hkv, Sk, D); }

int ref_bq(void) { return BQ; }

int ref_main(int argc, char **argv) { return flash_ref_main(argc, argv); }
