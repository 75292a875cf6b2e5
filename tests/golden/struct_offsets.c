/* struct_offsets.c -- prints the byte offset of every field of the weight-table
 * structs.  Compiled once against the reference's backends/model_types.h (to
 * make tests/golden/struct_offsets_ref.txt) and once against
 * include/ct_model_types.h (tests/test_abi_layout.py); the two must agree,
 * because the backend ABI passes these structs by pointer. */
#include <stdio.h>
#include <stddef.h>
#include MODEL_TYPES_HEADER

#define P(S, f) printf(#S "." #f " %zu\n", offsetof(S, f))

int main(void) {
    printf("sizeof.ELayer %zu\nsizeof.DLayer %zu\nsizeof.Weights %zu\n",
           sizeof(ELayer), sizeof(DLayer), sizeof(Weights));
    P(ELayer, ff1_lnw); P(ELayer, ff1_w2); P(ELayer, sa_lnw); P(ELayer, sa_pw);
    P(ELayer, sa_ow); P(ELayer, sa_pbu); P(ELayer, sa_pbv); P(ELayer, cv_lnw);
    P(ELayer, cv_dww); P(ELayer, cv_dwb); P(ELayer, cv_bnw); P(ELayer, cv_bnmean);
    P(ELayer, cv_bnvar); P(ELayer, cv_pw2b); P(ELayer, ff2_lnw); P(ELayer, out_lnb);
    P(DLayer, sa_lnw); P(DLayer, sa_ob); P(DLayer, ca_lnw); P(DLayer, ca_kw);
    P(DLayer, ca_ob); P(DLayer, ffn_lnw); P(DLayer, ffn_b2);
    P(Weights, s0w); P(Weights, sob); P(Weights, enc); P(Weights, prw); P(Weights, prb);
    P(Weights, etw); P(Weights, epw); P(Weights, elnw); P(Weights, elnb); P(Weights, dec);
    P(Weights, dlnw); P(Weights, dlnb); P(Weights, hdb);
    return 0;
}
