// relpos_umma.cuh -- encoder relative-position attention on the 5th-generation
// tensor cores (tcgen05 MMAs into TMEM), plain bf16 operands.  Included by
// encoder.cu inside namespace ct::enc (uses its D, H, DK, Batch).
//
// Per (utterance u, head h, 128-query tile q0) one CTA computes, for queries q
// of the tile and keys k < T = T_enc[u] (backends/cpu/backend.c:262-295):
//   score[q][k] = ((Q[q] + u_h) . K[k] + (Q[q] + v_h) . P[k - q + T_max - 1]) / sqrt(DK)
//   out[q]      = softmax_k(score[q]) . V
// The bias terms u_h . K[k] and v_h . P[m] are per-key / per-table-row scalars,
// computed once per layer for the whole batch (relpos_bias_dots).  Key tiles of
// 64, walked with an online softmax:
//   S  = Q . K_tile^T        (M 128, N 64,  K 160)  -> TMEM columns [0, 64)
//   BD = Q . P_band^T        (M 128, N 192, K 160)  -> TMEM columns [64, 256)
//        P_band = table rows m0 .. m0 + 191, m0 = k0 - q0 - 127 + T_max - 1:
//        every (q, k) pair of the tile has its relative row inside the band.
//   O += probs . V_tile      (M 128, N 160, K 64)   -> TMEM columns [256, 416)
// TMEM lane = query row, so each softmax thread owns one whole score row (no
// cross-thread reductions).  Row q needs BD at band column k - k0 + 127 - (q - q0):
// a window that slides with the row.  A warp loads the 96 band columns its 32
// rows can reach, and each thread shifts its 64 needed values into place with
// a five-stage register barrel shift (by 16, 8, 4, 2, 1 as the row offset's
// bits say).
// Operands: Q, K and P tiles by TMA with the 128-byte swizzle (K-major, three
// 64-column atoms cover DK = 160; the MMAs use the first 160 columns).  K is
// double-buffered; the band lives in a ring of four 64-row blocks (tile i
// reads blocks i, i + 1, i + 2, so each tile needs one new block, loaded a tile
// ahead; slots adjacent in memory go to one wider MMA).  V is transposed into a
// K-major [160 d][64 keys] tile by the staging warps; the probabilities are
// written by the softmax threads into TMEM (columns [416, 448), two bf16 per
// column) as the A operand of the P.V MMA.
// Warps: 0 TMA producer, 1 MMA issuer (TMEM owner), 2..5 softmax (TMEM lane
// quarters 2, 3, 0, 1), 6..9 V / bias staging.  Every wait is bounded.

constexpr int UQ = 128, UK = 64, UB = 192, UKA = 3;     // query tile, key tile, band rows, k atoms
constexpr int U_THREADS = 320;
constexpr uint32_t U_COL_S = 0, U_COL_BD = 64, U_COL_O = 256, U_COL_P = 416, U_TMEM_COLS = 512;
constexpr int U_SLOTS = 4;   // band ring slots: block b + 2 is loaded while tile b - 1 still reads slot (b - 2) % 4
static_assert(DK == 160, "the atom layout below assumes a 160-wide head");

struct RelposUmmaSmem {
    uint8_t q[UKA][UQ * 128];    // Q tile, three 64-column atoms (SW128, 1024-aligned)
    uint8_t k[2][UKA][UK * 128]; // K tiles (by tile parity)
    uint8_t p[UKA][U_SLOTS][UK * 128];   // band ring per atom: block b (table rows m_base + 64 b ..) in
                                         // slot b % 4; adjacent slots form one wider MMA operand
    uint8_t vt[DK * 128];        // V^T [160 d][64 keys]
    float uk[2][UK];             // u.K of the tile's keys (double-buffered by tile parity)
    float vp[2][UB];             // v.P of the band rows
    uint64_t qfull, kfull[2], pslot[U_SLOTS], kfree, sfull, sfree, vfull, pfull, pvdone;
    // bias tiles, one barrier per buffer: the staging warps may run a tile
    // ahead of the softmax, and one barrier would then alias its phases
    uint64_t bfull[2];
    uint32_t tmem_slot;
};

static_assert(sizeof(RelposUmmaSmem) + 1024 <= 227 * 1024, "rel-pos tile exceeds the shared memory of a CTA");

struct RelposUmmaArgs {
    const bf16 *qkv;      // [R3][3 D]: Q | K | V
    const float *ukg;     // [R3][H]: u_h . K[r]
    const float *vpg;     // [PL][H]: v_h . P[m]
    const int *qtile;     // utterance << 16 | first query row (128-row tiles)
    const int *r3_off;
    int T_max, PL;        // PL = 2 T_max - 1 table rows
    bf16 *out;            // [R3][D]
};

// Bounded wait that also gives up as soon as the device status word is set
// (by a wait of this launch that ran out, or an earlier error): a failed launch
// then ends within one wait budget instead of one per CTA and wait.
__device__ __forceinline__ bool u_wait(uint64_t *bar, uint32_t parity, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u) {
            if (*reinterpret_cast<volatile int *>(&g_ct_status) != 0) return false;
            if (globaltimer() - t0 > CT_WAIT_NS) {
                set_status(code);
                return false;
            }
        }
    }
}

// byte offset of element (row, col) in a K-major SW128 tile of 64-element rows
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((col >> 3) ^ row) & 7) << 4) + (col & 7) * 2);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16: A (M rows = TMEM lanes, K packed two
// bf16 per 32-bit column from a_tmem) is read from tensor memory.
__device__ __forceinline__ void mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
          "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
          "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
          "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
          "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
          "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
          "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
          "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
          "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
          "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
          "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 64 consecutive TMEM columns (32 per load) from taddr, one wait for all.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]),"=r"(r[1]),"=r"(r[2]),"=r"(r[3]),"=r"(r[4]),"=r"(r[5]),"=r"(r[6]),"=r"(r[7]),"=r"(r[8]),"=r"(r[9]),"=r"(r[10]),"=r"(r[11]),"=r"(r[12]),"=r"(r[13]),"=r"(r[14]),"=r"(r[15]),"=r"(r[16]),"=r"(r[17]),"=r"(r[18]),"=r"(r[19]),"=r"(r[20]),"=r"(r[21]),"=r"(r[22]),"=r"(r[23]),"=r"(r[24]),"=r"(r[25]),"=r"(r[26]),"=r"(r[27]),"=r"(r[28]),"=r"(r[29]),"=r"(r[30]),"=r"(r[31]),"=r"(r[32]),"=r"(r[33]),"=r"(r[34]),"=r"(r[35]),"=r"(r[36]),"=r"(r[37]),"=r"(r[38]),"=r"(r[39]),"=r"(r[40]),"=r"(r[41]),"=r"(r[42]),"=r"(r[43]),"=r"(r[44]),"=r"(r[45]),"=r"(r[46]),"=r"(r[47]),"=r"(r[48]),"=r"(r[49]),"=r"(r[50]),"=r"(r[51]),"=r"(r[52]),"=r"(r[53]),"=r"(r[54]),"=r"(r[55]),"=r"(r[56]),"=r"(r[57]),"=r"(r[58]),"=r"(r[59]),"=r"(r[60]),"=r"(r[61]),"=r"(r[62]),"=r"(r[63])
        : "r"(taddr + 0u), "r"(taddr + 32u)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 96 consecutive TMEM columns (32 per load) from taddr, one wait for all.
__device__ __forceinline__ void tmem_ld96(uint32_t taddr, float (&v)[96]) {
    uint32_t r[96];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%96];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%97];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95}, [%98];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]),"=r"(r[1]),"=r"(r[2]),"=r"(r[3]),"=r"(r[4]),"=r"(r[5]),"=r"(r[6]),"=r"(r[7]),"=r"(r[8]),"=r"(r[9]),"=r"(r[10]),"=r"(r[11]),"=r"(r[12]),"=r"(r[13]),"=r"(r[14]),"=r"(r[15]),"=r"(r[16]),"=r"(r[17]),"=r"(r[18]),"=r"(r[19]),"=r"(r[20]),"=r"(r[21]),"=r"(r[22]),"=r"(r[23]),"=r"(r[24]),"=r"(r[25]),"=r"(r[26]),"=r"(r[27]),"=r"(r[28]),"=r"(r[29]),"=r"(r[30]),"=r"(r[31]),"=r"(r[32]),"=r"(r[33]),"=r"(r[34]),"=r"(r[35]),"=r"(r[36]),"=r"(r[37]),"=r"(r[38]),"=r"(r[39]),"=r"(r[40]),"=r"(r[41]),"=r"(r[42]),"=r"(r[43]),"=r"(r[44]),"=r"(r[45]),"=r"(r[46]),"=r"(r[47]),"=r"(r[48]),"=r"(r[49]),"=r"(r[50]),"=r"(r[51]),"=r"(r[52]),"=r"(r[53]),"=r"(r[54]),"=r"(r[55]),"=r"(r[56]),"=r"(r[57]),"=r"(r[58]),"=r"(r[59]),"=r"(r[60]),"=r"(r[61]),"=r"(r[62]),"=r"(r[63]),"=r"(r[64]),"=r"(r[65]),"=r"(r[66]),"=r"(r[67]),"=r"(r[68]),"=r"(r[69]),"=r"(r[70]),"=r"(r[71]),"=r"(r[72]),"=r"(r[73]),"=r"(r[74]),"=r"(r[75]),"=r"(r[76]),"=r"(r[77]),"=r"(r[78]),"=r"(r[79]),"=r"(r[80]),"=r"(r[81]),"=r"(r[82]),"=r"(r[83]),"=r"(r[84]),"=r"(r[85]),"=r"(r[86]),"=r"(r[87]),"=r"(r[88]),"=r"(r[89]),"=r"(r[90]),"=r"(r[91]),"=r"(r[92]),"=r"(r[93]),"=r"(r[94]),"=r"(r[95])
        : "r"(taddr + 0u), "r"(taddr + 32u), "r"(taddr + 64u)
        : "memory");
#pragma unroll
    for (int i = 0; i < 96; ++i) v[i] = __uint_as_float(r[i]);
}

// u_h . K[r] and v_h . P[m] for every packed row r and table row m, all heads
// (fp32 sums of the bf16 hi (+ lo) planes).  One warp per row: lane l takes
// head l / 4, dims (l % 4) * 40 .. + 40 as five 16-byte loads, sums them in
// order, and the four lanes of a head add their sums by two butterfly steps.
static_assert(H * 4 == 32 && DK == 4 * 40, "four lanes per head, 40 dims each");
__device__ __forceinline__ float dot8_bf16(const uint4 &a, const uint4 &w, float acc) {
    const __nv_bfloat162 *a2 = reinterpret_cast<const __nv_bfloat162 *>(&a);
    const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 x = __bfloat1622float2(a2[i]), y = __bfloat1622float2(w2[i]);
        acc += y.x * x.x;
        acc += y.y * x.y;
    }
    return acc;
}
__global__ void __launch_bounds__(256) relpos_bias_dots(const bf16 *qkv_h, const bf16 *qkv_l, const bf16 *P_h,
                                                        const bf16 *P_l, int R3, int PL, const bf16 *pbu,
                                                        const bf16 *pbv, float *ukg, float *vpg) {
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= R3 + PL) return;
    const bool is_k = w < R3;
    const int r = is_k ? w : w - R3;
    const int h = lane >> 2, d0 = h * DK + (lane & 3) * 40;
    const size_t base = (is_k ? (size_t)r * 3 * D + D : (size_t)r * D) + d0;
    const uint4 *hi = reinterpret_cast<const uint4 *>((is_k ? qkv_h : P_h) + base);
    const bf16 *lo_p = is_k ? qkv_l : P_l;
    const uint4 *bias = reinterpret_cast<const uint4 *>((is_k ? pbu : pbv) + d0);
    uint4 x[5], bv[5];
#pragma unroll
    for (int j = 0; j < 5; ++j) { x[j] = hi[j]; bv[j] = bias[j]; }
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 5; ++j) acc = dot8_bf16(x[j], bv[j], acc);
    if (lo_p) {
        const uint4 *lo = reinterpret_cast<const uint4 *>(lo_p + base);
#pragma unroll
        for (int j = 0; j < 5; ++j) acc = dot8_bf16(lo[j], bv[j], acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if ((lane & 3) == 0) (is_k ? ukg : vpg)[(size_t)r * H + h] = acc;
}

__global__ void __launch_bounds__(U_THREADS, 1) relpos_umma(const __grid_constant__ CUtensorMap tmQ,
                                                            const __grid_constant__ CUtensorMap tmK,
                                                            const __grid_constant__ CUtensorMap tmP,
                                                            const RelposUmmaArgs a) {
    extern __shared__ __align__(1024) uint8_t umma_raw[];
    RelposUmmaSmem &sm =
        *reinterpret_cast<RelposUmmaSmem *>((reinterpret_cast<uintptr_t>(umma_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const int wq = a.qtile[blockIdx.x];
    const int u = wq >> 16, q0 = wq & 0xFFFF;
    const int base = a.r3_off[u];
    const int T = a.r3_off[u + 1] - base;
    const int Tm = a.T_max;
    const int nkt = (T + UK - 1) / UK;   // >= 1: the host lists tiles of non-empty utterances only
    if (threadIdx.x == 0) {
        mbar_init(&sm.qfull, 1);
        for (int b = 0; b < 2; ++b) mbar_init(&sm.kfull[b], 1);
        for (int b = 0; b < U_SLOTS; ++b) mbar_init(&sm.pslot[b], 1);
        mbar_init(&sm.kfree, 1);
        mbar_init(&sm.sfull, 1);
        mbar_init(&sm.sfree, 4);
        mbar_init(&sm.bfull[0], 128);
        mbar_init(&sm.bfull[1], 128);
        mbar_init(&sm.vfull, 128);
        mbar_init(&sm.pfull, 128);
        mbar_init(&sm.pvdone, 1);
        fence_mbar_init();
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmP);
    }
    if (warp == 1) { tmem_alloc(&sm.tmem_slot, U_TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_slot;
    const int mb0 = -q0 - (UQ - 1) + Tm - 1;   // first table row of band block 0 (tile 0's band start)

    if (warp == 0) {
        // ------------------------------------------------------------- producer
        if (lane == 0) {
            auto load_k = [&](int i) {   // K tile i into buffer i & 1
                mbar_expect_tx(&sm.kfull[i & 1], UKA * UK * 128);
                for (int kb = 0; kb < UKA; ++kb)
                    tma_load_2d(sm.k[i & 1][kb], &tmK, &sm.kfull[i & 1], D + h * DK + kb * 64, base + i * UK);
            };
            auto load_p = [&](int b) {   // band block b into slot b % 4
                const int sl = b % U_SLOTS;
                mbar_expect_tx(&sm.pslot[sl], UKA * UK * 128);
                for (int kb = 0; kb < UKA; ++kb)
                    tma_load_2d(sm.p[kb][sl], &tmP, &sm.pslot[sl], h * DK + kb * 64, mb0 + b * UK);
            };
            mbar_expect_tx(&sm.qfull, UKA * UQ * 128);
            for (int kb = 0; kb < UKA; ++kb) tma_load_2d(sm.q[kb], &tmQ, &sm.qfull, h * DK + kb * 64, base + q0);
            load_k(0);
            for (int b = 0; b < 3; ++b) load_p(b);
            if (nkt > 1) { load_k(1); load_p(3); }
            for (int i = 1; i + 1 < nkt; ++i) {
                // S / BD of tile i - 1 complete: band block i - 1's slot (block
                // i + 3's) and K buffer (i + 1) & 1 (tile i - 1's) are free
                if (!u_wait(&sm.kfree, (uint32_t)(i - 1) & 1u, CT_STATUS_TIMEOUT_FREE)) break;
                load_k(i + 1);
                load_p(i + 3);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t id_o = idesc_bf16(UQ, DK);
            bool ok = u_wait(&sm.qfull, 0, CT_STATUS_TIMEOUT_TMA);
            // Q . X^T over the 160 head columns (three atoms, the last one half used)
            // for an X of n rows whose atom kb starts at x(kb)
            auto qx = [&](uint32_t dcol, int n, auto x) {
                const uint32_t id = idesc_bf16(UQ, n);
#pragma unroll
                for (int kb = 0; kb < UKA; ++kb) {
                    const uint64_t qd = sw128_desc(smem_u32(sm.q[kb]));
                    const uint64_t xd = sw128_desc(smem_u32(x(kb)));
                    const int nks = kb < UKA - 1 ? 4 : (DK - 128) / 16;   // 160 = 64 + 64 + 32
                    for (int k = 0; k < nks; ++k)
                        mma_bf16(tmem + dcol, qd + 2 * k, xd + 2 * k, id, (kb | k) ? 1u : 0u);
                }
            };
            for (int i = 0; i <= nkt && ok; ++i) {
                if (i < nkt) {
                    // S and BD of tile i once K_i landed and the softmax threads have
                    // read tile i - 1 out of TMEM
                    ok = u_wait(&sm.kfull[i & 1], (uint32_t)(i >> 1) & 1u, CT_STATUS_TIMEOUT_TMA);
                    if (ok && i > 0) ok = u_wait(&sm.sfree, (uint32_t)(i - 1) & 1u, CT_STATUS_TIMEOUT_MMA);
                    if (!ok) break;
                    // band blocks i, i + 1, i + 2 (loaded a tile ahead): wait for the ones not seen yet
                    for (int b = (i == 0 ? 0 : i + 2); b <= i + 2 && ok; ++b)
                        ok = u_wait(&sm.pslot[b % U_SLOTS], (uint32_t)(b / U_SLOTS) & 1u, CT_STATUS_TIMEOUT_TMA);
                    if (!ok) break;
                    tc_fence_after();
                    const int kbuf = i & 1, r = i % U_SLOTS;
                    qx(U_COL_S, UK, [&](int kb) { return sm.k[kbuf][kb]; });
                    // band positions 0, 1, 2 are slots r, r + 1, r + 2 (mod 4); runs of
                    // slots adjacent in memory go as one MMA
                    if (r <= 1) {
                        qx(U_COL_BD, 3 * UK, [&](int kb) { return sm.p[kb][r]; });
                    } else if (r == 2) {
                        qx(U_COL_BD, 2 * UK, [&](int kb) { return sm.p[kb][2]; });
                        qx(U_COL_BD + 2 * UK, UK, [&](int kb) { return sm.p[kb][0]; });
                    } else {
                        qx(U_COL_BD, UK, [&](int kb) { return sm.p[kb][3]; });
                        qx(U_COL_BD + UK, 2 * UK, [&](int kb) { return sm.p[kb][0]; });
                    }
                    mma_commit(&sm.sfull);
                    mma_commit(&sm.kfree);
                }
                if (i > 0) {
                    // P.V of tile i - 1
                    const int j = i - 1;
                    ok = u_wait(&sm.pfull, (uint32_t)j & 1u, CT_STATUS_TIMEOUT_MMA) &&
                         u_wait(&sm.vfull, (uint32_t)j & 1u, CT_STATUS_TIMEOUT_TMA);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t vd = sw128_desc(smem_u32(sm.vt));
#pragma unroll
                    for (int k = 0; k < UK / 16; ++k)   // A = the probabilities in TMEM (16 bf16 = 8 columns a step)
                        mma_bf16_ta(tmem + U_COL_O, tmem + U_COL_P + 8u * k, vd + 2 * k, id_o, (j | k) ? 1u : 0u);
                    mma_commit(&sm.pvdone);
                }
            }
        }
    } else if (warp >= 6) {
        // ------------------------------------------ V^T and bias staging (128 threads)
        // Each tile's global loads are issued one tile ahead into registers,
        // so only the shared-memory stores wait for the previous P.V.
        const int t = threadIdx.x - 192;
        const int ka = 2 * (t & 31), cq = t >> 5;   // keys (ka, ka + 1), chunks cq, cq + 4, ...
        constexpr int NCH = DK / 8 / 4;              // 16-byte chunks per key and thread
        uint4 va[NCH], vb[NCH];
        float uk_r = 0.0f, vp_r0 = 0.0f, vp_r1 = 0.0f;
        auto load_tile = [&](int i) {
            const int k0 = i * UK, m0 = k0 - q0 - (UQ - 1) + Tm - 1;
            const bf16 *src = a.qkv + (size_t)(base + k0 + ka) * 3 * D + 2 * D + h * DK;
            const bool oka = k0 + ka < T, okb = k0 + ka + 1 < T;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const int ch = cq + 4 * c;
                va[c] = oka ? *reinterpret_cast<const uint4 *>(src + ch * 8) : make_uint4(0, 0, 0, 0);
                vb[c] = okb ? *reinterpret_cast<const uint4 *>(src + (size_t)3 * D + ch * 8) : make_uint4(0, 0, 0, 0);
            }
            uk_r = (t < UK && k0 + t < T) ? a.ukg[(size_t)(base + k0 + t) * H + h] : 0.0f;
            const int m1 = m0 + t, m2 = m0 + t + 128;
            vp_r0 = (m1 >= 0 && m1 < a.PL) ? a.vpg[(size_t)m1 * H + h] : 0.0f;
            vp_r1 = (t + 128 < UB && m2 >= 0 && m2 < a.PL) ? a.vpg[(size_t)m2 * H + h] : 0.0f;
        };
        load_tile(0);
        for (int i = 0; i < nkt; ++i) {
            // bias buffer i & 1 was last read by the softmax of tile i - 2, which
            // finished before P.V of tile i - 2 (seen complete last iteration)
            float *ukb = sm.uk[i & 1], *vpb = sm.vp[i & 1];
            if (t < UK) ukb[t] = uk_r;
            vpb[t] = vp_r0;
            if (t + 128 < UB) vpb[t + 128] = vp_r1;
            mbar_arrive(&sm.bfull[i & 1]);
            // V^T of tile i overwrites tile i - 1's, read by its P.V
            if (i > 0 && !u_wait(&sm.pvdone, (uint32_t)(i - 1) & 1u, CT_STATUS_TIMEOUT_MMA)) break;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const int ch = cq + 4 * c;
                const uint32_t wa[4] = {va[c].x, va[c].y, va[c].z, va[c].w};
                const uint32_t wb[4] = {vb[c].x, vb[c].y, vb[c].z, vb[c].w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    // d = ch * 8 + e: (V[ka][d], V[ka + 1][d]) as one 32-bit pair
                    const uint32_t lo16 = (wa[e >> 1] >> ((e & 1) * 16)) & 0xFFFFu;
                    const uint32_t hi16 = (wb[e >> 1] >> ((e & 1) * 16)) & 0xFFFFu;
                    *reinterpret_cast<uint32_t *>(sm.vt + sw128_off(ch * 8 + e, ka)) = lo16 | (hi16 << 16);
                }
            }
            fence_proxy_async_smem();   // the MMA reads V^T through the async proxy
            mbar_arrive(&sm.vfull);
            if (i + 1 < nkt) load_tile(i + 1);
        }
    } else {
        // ------------------------------------------------- softmax (warps 2..5)
        // The exponent reference m of a row moves only when the tile maximum
        // exceeds it by more than U_RESCALE (probabilities then stay below
        // e^U_RESCALE), so the O accumulator is rescaled in TMEM only on
        // those tiles; the final division by l is exact either way.
        constexpr float U_RESCALE = 8.0f;
        const int qw = warp & 3;
        const int ql = qw * 32 + lane;           // query row in the tile = TMEM lane
        const uint32_t trow = tmem + ((uint32_t)(qw * 32) << 16);
        const int c0w = 96 - 32 * qw;            // first band column this warp reads
        const int woff = 31 - lane;              // loaded column index of this row's key 0
        const float scale = 1.0f / sqrtf((float)DK);
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int i = 0; i < nkt; ++i) {
            const int k0 = i * UK;
            ok = ok && u_wait(&sm.sfull, (uint32_t)i & 1u, CT_STATUS_TIMEOUT_MMA) &&
                 u_wait(&sm.bfull[i & 1], (uint32_t)(i >> 1) & 1u, CT_STATUS_TIMEOUT_TMA);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            const float *ukb = sm.uk[i & 1], *vpb = sm.vp[i & 1];
            // BD: the 96 band columns this warp reaches, + v.P of their table rows,
            // shifted left by this row's offset woff so that bd[j] is key k0 + j's
            float bd[96];
            tmem_ld96(trow + U_COL_BD + (uint32_t)c0w, bd);
#pragma unroll
            for (int jj = 0; jj < 96; ++jj) bd[jj] += vpb[c0w + jj];
#pragma unroll
            for (int j = 0; j < 80; ++j) bd[j] = (woff & 16) ? bd[j + 16] : bd[j];
#pragma unroll
            for (int j = 0; j < 72; ++j) bd[j] = (woff & 8) ? bd[j + 8] : bd[j];
#pragma unroll
            for (int j = 0; j < 68; ++j) bd[j] = (woff & 4) ? bd[j + 4] : bd[j];
#pragma unroll
            for (int j = 0; j < 66; ++j) bd[j] = (woff & 2) ? bd[j + 2] : bd[j];
#pragma unroll
            for (int j = 0; j < 64; ++j) bd[j] = (woff & 1) ? bd[j + 1] : bd[j];
            float sc[UK];
            tmem_ld64(trow + U_COL_S, sc);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.sfree);   // S / BD may be overwritten
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < UK; ++j) {
                float x = (sc[j] + ukb[j] + bd[j]) * scale;
                if (k0 + j >= T) x = -INFINITY;
                sc[j] = x;
                mx = fmaxf(mx, x);
            }
            // mx is finite: key k0 < T
            const bool move = mx > m + U_RESCALE;      // always on the first tile (m = -inf)
            const float mn = move ? mx : m;
            const float corr = move ? __expf(m - mn) : 1.0f;   // 0 on the first tile
            float ls = 0.0f;
#pragma unroll
            for (int j = 0; j < UK; ++j) {
                const float pj = __expf(sc[j] - mn);
                sc[j] = pj;
                ls += pj;
            }
            l = l * corr + ls;
            m = mn;
            if (i > 0) {
                // P.V of tile i - 1 done: O may be rescaled and the probability tile reused
                ok = u_wait(&sm.pvdone, (uint32_t)(i - 1) & 1u, CT_STATUS_TIMEOUT_MMA);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc_fence_after();
                if (__any_sync(0xffffffffu, move)) {
#pragma unroll 1
                    for (int c = 0; c < DK; c += 32) {
                        float o32[32];
                        tmem_ld32(trow + U_COL_O + (uint32_t)c, o32);
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) o32[jj] *= corr;
                        tmem_st32(trow + U_COL_O + (uint32_t)c, o32);
                    }
                }
            }
            // probabilities -> the P.V MMA's A operand in TMEM: row ql, keys 2c, 2c + 1
            // packed in column c as bf16 (lower key in the low half)
            {
                float pk[32];
#pragma unroll
                for (int c = 0; c < UK / 2; ++c) {
                    const __nv_bfloat162 pr2 = __floats2bfloat162_rn(sc[2 * c], sc[2 * c + 1]);
                    pk[c] = __uint_as_float(*reinterpret_cast<const uint32_t *>(&pr2));
                }
                tmem_st32(trow + U_COL_P, pk);
            }
            tc_fence_before();
            mbar_arrive(&sm.pfull);
        }
        // ------------------------------------------------------------ epilogue
        if (ok) ok = u_wait(&sm.pvdone, (uint32_t)(nkt - 1) & 1u, CT_STATUS_TIMEOUT_MMA);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
            tc_fence_after();
            const float inv = 1.0f / l;
            const bool store = q0 + ql < T;
            bf16 *dst = a.out + (size_t)(base + q0 + ql) * D + h * DK;
#pragma unroll 1
            for (int c = 0; c < DK / 32; ++c) {
                float v[32];
                tmem_ld32(trow + U_COL_O + (uint32_t)(32 * c), v);
                if (store) {
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        uint32_t w4[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 o2 =
                                __floats2bfloat162_rn(v[8 * g + 2 * e] * inv, v[8 * g + 2 * e + 1] * inv);
                            w4[e] = *reinterpret_cast<const uint32_t *>(&o2);
                        }
                        *reinterpret_cast<uint4 *>(dst + 32 * c + 8 * g) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, U_TMEM_COLS);
}
