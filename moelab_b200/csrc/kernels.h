// Internal kernel argument blocks and declarations (not part of the C ABI).
#pragma once
#include <cuda.h>  // CUtensorMap
#include <cuda_runtime.h>
#include <stdint.h>

namespace moeb {

enum { FMT_Q4 = 0, FMT_FP4 = 1 };

struct RouterArgs {
    const uint16_t *x;     // [T][d] bf16
    const uint16_t *wg;    // [E][d] bf16 gate
    const uint16_t *bias;  // [E] bf16 or null
    int T, d, E, k, norm;
    int ns;  // shared experts: ids E .. E + ns - 1 appended to every token with weight 1 (slots per token k + ns)
    float scale;
    float *logits;  // [T][E] fp32 (workspace or caller buffer)
    int *idx;       // [T][k]
    float *wts;     // [T][k]
    float *xsum;    // [T][d/64] or null
    unsigned *cnt;      // [ceil(T/TPB)] zero-initialised, self-resetting
    unsigned *cnt_all;  // [1] zero-initialised, self-resetting
    // tile mode (null tiles = slot mode)
    int NT;
    int4 *tiles;
    int *ntiles;
    int *sorted;
    unsigned *err;
};

struct PrepArgs {
    const uint16_t *x;
    const int *idx;
    int T, d, E, k;
    int xs;  // x row stride in bf16 elements (d, or d + 8 for expert-parallel rows with their tail)
    // expert-parallel rows (k == 1): each row's tail {local expert, weight bits} is unpacked into these
    int *idx_w;
    float *wts_w;
    // peer-memory exchange: rows arrive in blocks of C rows per source (this call's block size); rflag[src] ==
    // *epoch once source src has written its rcnt[src] rows (null: rows are all valid)
    const unsigned *rflag;
    const int *rcnt;
    const unsigned *epoch;
    const unsigned long long *wait_ns;  // the exchange's wait limit (0 = the 2 s default)
    int C;
    float *xsum;
    unsigned *cnt_all;
    int NT;
    int4 *tiles;
    int *ntiles;
    int *sorted;
    unsigned *err;
    int *counts, *offsets;  // optional [E] outputs of the tile builder (per-expert slot counts, prefix offsets)
};

// Expert weights of one projection in the B200 layout.
struct QProj {
    const uint32_t *q;   // packed codes [E][N][K/8]
    const uint32_t *sb;  // int4: scale|bias [E][N][K/64]; mxfp4: e8m0 bytes [E][N][K/32]
};

struct ExpArgs {
    const uint16_t *x;  // [T][xs] bf16 (the first d values of each row are the activations)
    int xs;             // x row stride in bf16 elements
    const float *xsum;  // [T][d/64]
    QProj g, u, dn;
    const float *bg, *bu, *bd;  // optional expert biases [E][f], [E][f], [E][d]
    const int *idx;             // [T*k]
    const float *wts;           // [T*k]
    const int4 *tiles;          // tile mode: (expert, start, n, 0)
    const int *ntiles;
    const int *sorted;
    uint16_t *h;           // [TK][f] bf16
    float *hsum;           // [TK][f/16] fp32 (sums of 16 consecutive bf16 h values)
    float *yp;             // [TK][d] fp32 weighted per-slot outputs
    unsigned *ycnt;        // [T][d/16] zero-initialised, self-resetting
    const uint16_t *residual;  // optional [T][d]
    uint16_t *y;               // [T][d] bf16
    unsigned *err;
    int T, d, f, E, k, act, tile_mode;
    int dn_prefetch;  // gate/up pulls the down weights of its expert into L2
    int early_ids;    // down reads its routing and issues its first weight loads before waiting for gate/up
    int fmt;          // FMT_Q4 or FMT_FP4
    int h_kperm;      // gate/up writes h with the 64-group k order permuted for a TMEM-operand tensor-core down
    int slot_out;     // 1: down stops after writing the weighted per-slot outputs yp (caller's buffer), no combine
    // peer-memory exchange: slot s's weighted row goes to (float *)(ypeers[s / C] + yoff) + (me * C + s % C) * d
    // (C = this call's block size), this rank's return block in the owner's buffer, instead of yp; the writing
    // warps fence at system scope
    unsigned char *const *ypeers;
    size_t yoff;
    int C, me;
    // warp-specialized kernels: 2-D tensor maps over each projection's codes (uint64 elements) and scale|bias
    // words (uint32), viewed as [row blocks of all experts][K/64 groups x 512 B | 64 B] ([0] gate, [1] up,
    // [2] down); a box is RBC row blocks x SG groups (RBC rows of SG*512 | SG*64 contiguous bytes), so one
    // copy per array and projection fills a pipeline stage
    CUtensorMap tmq[3], tmsb[3];
    // tensor-core kernels: 2-D map over the expert-sorted activation rows of the launch (x gathered for gate/up,
    // h for down), box 64 k x NT rows, 128-byte swizzle
    CUtensorMap tmx;
};

// Per-rank buffer of the peer-memory exchange (one allocation, mapped by every rank of the group):
//   epoch counter, error word, a grid counter and the wait limit (u64 ns, 0 = 2 s), rflag[P] / rcnt[P] (written
//   by the sources), bflag[P] (written by the expert ranks), rows [P][C][d + 8] bf16 (source blocks), back [P][C][d]
//   fp32 (return blocks).
struct P2PLayout {
    size_t epoch, err, ctr, wait, rflag, rcnt, bflag, rows, back, total;
};
__host__ __device__ inline P2PLayout p2p_layout(int P, int C, int d) {
    P2PLayout L;
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    L.epoch = 0;
    L.err = 64;
    L.ctr = 128;
    L.wait = 192;
    L.rflag = 256;
    L.rcnt = L.rflag + up(4 * (size_t)P);
    L.bflag = L.rcnt + up(4 * (size_t)P);
    L.rows = L.bflag + up(4 * (size_t)P);
    L.back = L.rows + up((size_t)P * C * (d + 8) * 2);
    L.total = L.back + up((size_t)P * C * d * 4);
    return L;
}

// Expert-parallel dispatch plan / pack / combine (csrc/ep.cu).
struct EPArgs {
    const uint16_t *x;    // [T][d] bf16
    const int *idx;       // [T*k] global expert ids
    const float *wts;     // [T*k]
    int T, d, k, E, P;    // P ranks own E/P consecutive experts each
    int *send_counts;     // [P]
    int *slot_pos;        // [T*k] row of each slot in the send buffer, -1 = dropped (invalid id)
    uint16_t *rows;       // [T*k][d + 8] send rows: x of the slot's token, then {local expert, weight, 0, 0}
    unsigned *err;
    // peer-memory exchange (C > 0, the buffers' capacity in rows per source): this call's blocks hold Cs rows
    // (Cs <= C), slot_pos is in block layout (dst * Cs + rank inside dst), rows are written into peers[dst]'s
    // source block `me`; self = this rank's exchange buffer (epoch, counters)
    int C, Cs, me;
    unsigned char *const *peers;
    unsigned char *self;
};
__global__ void k_ep_plan(EPArgs a);
__global__ void k_ep_pack(EPArgs a);
__global__ void k_combine(const float *yp, int T, int d, int k, const uint16_t *residual, uint16_t *y);
// Single-kernel decode layer (decode.cu): DEC_NW consumer warps + 1 producer warp per CTA, one CTA per SM.
constexpr int DEC_NW = 15, DEC_THREADS = 32 * (DEC_NW + 1), DEC_CG = 8;  // 16 warps: 128 registers each
struct DecodePlan {
    int NW, CGd, CGf;      // consumer warps, 64-groups per item (gate/up: a divisor of d/64, down: of f/64)
    int NCd, NCf;          // items per (gate/up unit, projection) and per down unit
    int NSLOT, slot_bytes; // ring of bulk-copy slots
    int NSL;               // h staging rows (distinct down slots of one CTA)
    int max_gu_units, max_dn_units;
    int nR;                // CTAs computing logits
    // dynamic shared memory offsets (bytes)
    int o_ring, o_bar, o_x, o_xsum, o_idx, o_wts, o_part, o_ucnt, o_h, o_hstate, total;
};
struct DecodeArgs {
    ExpArgs a;
    RouterArgs r;     // r.wg == null: ids given in a.idx / a.wts
    DecodePlan p;
    unsigned *arr;    // arrivals of the call's CTAs (zeroed; the last arrival resets it)
    unsigned *gen;    // generation word: advanced once per call by the last arrival; the call's record tag
    unsigned long long *hrec;  // [T*k][f] records {tag, bf16 h}
    unsigned long long *yrec;  // [T*k][d] records {tag, fp32 weighted slot output}
};
template <int FMT>
__global__ void k_decode(const __grid_constant__ DecodeArgs A);
__global__ void k_ep_send(EPArgs a);
__global__ void k_ep_signal(unsigned char *const *peers, unsigned char *self, int P, int C, int d, int me);
__global__ void k_ep_combine_p2p(const unsigned char *self, const int *slot_pos, int P, int C, int T, int d, int k,
                                 const uint16_t *residual, uint16_t *y, unsigned *err);
__global__ void k_ep_combine(const float *back, const int *slot_pos, int T, int d, int k, const uint16_t *residual,
                             uint16_t *y);

template <int TPB, int JMAX, int U, bool PRE>
__global__ void k_router(RouterArgs a);
template <int TW, int EW, int JMAX>
__global__ void k_router_t(RouterArgs a);
template <int JMAX>
__global__ void k_router_cl(RouterArgs a);
__global__ void k_prep(PrepArgs a);
size_t tiles_smem(int threads, int E, long TK, size_t cap);

__global__ void k_q4_quantize(const uint16_t *w, long rows, long K, uint32_t *qw, uint32_t *sb);
__global__ void k_q4_dequant(const uint32_t *qw, const uint32_t *sb, long rows, long K, float *out);
__global__ void k_q4_from_mlx(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases, long rows, long K,
                              uint32_t *qw, uint32_t *sb);
__global__ void k_fp4_quantize(const uint16_t *w, long rows, long K, uint32_t *qw, uint8_t *sc);
__global__ void k_fp4_dequant(const uint32_t *qw, const uint8_t *sc, long rows, long K, float *out);
__global__ void k_fp4_from_mlx(const uint32_t *wq, const uint8_t *scales, long rows, long K, uint32_t *qw,
                               uint8_t *sc);

template <int FMT, int KS, int GPW>
__global__ void k_gate_up_slots(ExpArgs a);
template <int FMT, int KS, int GPW>
__global__ void k_down_slots(ExpArgs a);
template <int FMT, int KS, int VW, int GPW>
__global__ void k_down_tok(ExpArgs a);
size_t down_tok_smem(int k, int f, int ks);
template <int FMT, int NT8, int GPW>
__global__ void k_gate_up_tiles_reg(ExpArgs a);
template <int FMT, int NT8, int GPW>
__global__ void k_down_tiles_reg(ExpArgs a);
template <int FMT, int NT8, int RBC, int SG, int NS, bool DOWN, int MB>
__global__ void k_experts_ws(const __grid_constant__ ExpArgs a);
template <int FMT, int NT, int NR, int NA, int NX, int ACC, bool DOWN>
__global__ void k_experts_tc(const __grid_constant__ ExpArgs a);
template <int FMT, int NT, int NR, int NS, int ACC, bool DOWN, int SGK>
__global__ void k_experts_tca(const __grid_constant__ ExpArgs a);
// The tcgen05 expert kernel for (format, tile size 32 / 64 / 128 / 256, projection): entry, block size and
// dynamic shared memory (fn == nullptr for an unsupported tile size).
struct TcInfo {
    void (*fn)(ExpArgs);
    int threads;
    size_t smem;
    bool tmem_a;  // A operand in TMEM: activations in the permuted 64-group k order
    int sg;       // 64-groups per pipeline stage (the weight tensor maps' box width)
};
TcInfo experts_tc_info(int fmt, int nt, bool down);
__global__ void k_gather_rows(const uint16_t *x, const int *sorted, int TK, int k, int d, int xstride, int perm,
                              uint16_t *xs);
size_t experts_ws_smem(int nt8, int rbc, int sg, int ns, bool down, int fmt);


size_t zero_region_bytes(size_t ws_bytes, int d, int f, int E, int k);
void decode_record_span(size_t ws_bytes, int d, int f, int E, int k, size_t *off, size_t *len);
void set_error(const char *msg);  // message returned by moeb_last_error()

}  // namespace moeb
