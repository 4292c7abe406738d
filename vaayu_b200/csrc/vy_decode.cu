// vy_decode.cu -- the bandwidth-bound expert layer: a token-batched int4 dequant GEMV.
//
// Work is cut so that every routed expert's packed weights cross HBM exactly once per call,
// whatever the number of tokens routed to it:
//
//   gate_up_kernel  one warp = 16 rows of one live expert's gate AND up projections, all of
//                   the expert's tokens (up to 8*NB per pass).  Codes stream through a
//                   per-warp cp.async ring (128 K elements per stage, kGuDepth stages in
//                   flight); each thread dequantises the 16-byte chunks it copied itself into
//                   activation-dtype pairs with two packed ops per pair (sub, mul: the
//                   reference's exact rounding of every weight) and feeds them to m16n8k16
//                   tensor-core fragments (fp32 accumulate) whose N dimension is the tokens.
//                   Epilogue: g, u, SiLU, product, each rounded to the activation dtype, into
//                   h (stored in the pair-permuted order the down kernel reads).  A call with
//                   few units per warp splits each unit's K range over 2-8 warps: they store
//                   their stages' partial dots and the last to finish adds all of them in stage
//                   order, so the result does not depend on the split.
//   down_kernel     one warp = 16 output rows of the down projection for one pass of a live
//                   expert (units dealt pass-major over every warp), y = h . Wd^T for every
//                   routed row, times the routing weight, into fp32 contributions by row id.
//   combine         (vy_route.cu) each token's contributions summed in ascending expert id,
//                   then slot -- no atomics on the sums.
//
// Two other decompositions of the same units serve small calls (all three give the same bits):
//   row_gate_up_kernel / row_down_kernel   at most 16 routed rows: one CTA per (routed row,
//                   16-row tile), no routing plan, the combine fused into the down kernel;
//   pass_gate_up_kernel / pass_down_kernel 17-64 routed rows over many experts: the planned
//                   passes, one CTA per (pass, tile) whose warps share the K range.
//
// The dequantised operand never touches shared memory, which is what keeps this path on HBM
// bandwidth: a tcgen05 GEMM would have to write every dequantised weight to shared memory and
// read it back (2 x 2 bytes per int4 weight), more shared-memory traffic per SM than the SM has
// at HBM rate, and its smallest tile (M = 64 / 128) would be mostly empty at 1-8 tokens.
#include "vy_moe.cuh"

namespace vy {
namespace {

#ifndef VY_GU_DEPTH
#define VY_GU_DEPTH 6
#endif
#ifndef VY_DN_DEPTH
#define VY_DN_DEPTH 8
#endif
#ifndef VY_GU_WARPS
#define VY_GU_WARPS 8
#endif
constexpr int kWarps = 8;                 // down-projection warps per CTA
constexpr int kGuWarps = VY_GU_WARPS;     // gate/up warps per CTA (two CTAs per SM)
constexpr int kStageK = 128;             // K elements of one row per pipeline stage (64 bytes of codes)
constexpr int kGuDepth = VY_GU_DEPTH;    // gate/up ring: stages in flight per warp (2 KB each)
constexpr int kDnDepth = VY_DN_DEPTH;    // down ring: stages in flight per warp (1 KB each)
constexpr int kTileRows = 16;
// Resident down-projection CTAs per SM by column blocks: the register bound each variant meets
// without spilling (its 64 KB shared-memory ring fits three); the down grid is one such wave.
constexpr int kDnBlocksPerSm[5] = {0, 3, 2, 0, 1};

struct GateUpParams {
    int hidden, inter, gs_shift, top_k;
    int64_t w_off[2], s_off[2], z_off[2];   // gate, up
    const PassEntry* passes;
    const int32_t* unit_start;               // unit_start[n_live] = number of passes
    int32_t* counters;                       // [0] n_live, [2] error flags
    const uint16_t* x_perm;
    uint16_t* h_perm;
    uint16_t* h_out;
    int max_passes;       // host side: the largest pass count the call can have (grid bound)
    int k_splits;         // warps sharing one unit's K range (1: none)
    float* partial;       // k_splits > 1: [unit][stage][lane][8 NB] per-stage partial dots
    int32_t* tickets;     // k_splits > 1: [unit] finished splits, zeroed by the plan kernel
};

struct DownParams {
    int hidden, inter, gs_shift, top_k;
    int64_t w_off, s_off, z_off;
    const PassEntry* passes;
    const int32_t* unit_start;
    int32_t* counters;
    const uint16_t* h_perm;
    const void* weights;
    int w_dtype;
    bool w_round;
    int64_t w_tok_stride, w_slot_stride;
    const int32_t* w_index;
    float* ybuf_g;        // [n][hidden] weighted contributions, by row id (token * top_k + slot)
};

// What a warp needs about one unit of work: a pass of a live expert (and, for gate/up, a 16-row
// tile of it).  Loaded one unit ahead of its use, so its latency hides behind the current unit.
template <int NB>
struct UnitInfo {
    const int32_t* pk;
    const void* sc;
    const int32_t* zp;
    int ncols;
    int tile;
    int split;         // gate/up with split K: which share of the unit's K range
    int unit;          // gate/up with split K: pass * tiles + tile
    int col_row[NB];   // row id of this lane's column (cb * 8 + g) in each block, -1 if none
    bool ok;
};

// The per-warp hand-off of unit descriptions from the issue side to the consuming side: the
// warp-uniform part once, the row ids per column.  Q slots cover the issue side's lookahead
// (kDepth - 1 stages, so at most kDepth - 1 units when a unit has a single stage).
template <int NB, int Q, int W = kWarps>
struct UnitQueue {
    struct Head {
        const int32_t* pk;
        const void* sc;
        const int32_t* zp;
        int ncols, tile, split, unit, ok;
    } head[W][Q];
    int rows[W][Q][NB * 8];

    __device__ __forceinline__ void put(int warp, int slot, int lane, int g, const UnitInfo<NB>& u) {
        if (lane == 0) head[warp][slot] = Head{u.pk, u.sc, u.zp, u.ncols, u.tile, u.split, u.unit, u.ok};
        if ((lane & 3) == 0)
#pragma unroll
            for (int cb = 0; cb < NB; ++cb) rows[warp][slot][cb * 8 + g] = u.col_row[cb];
    }
    __device__ __forceinline__ UnitInfo<NB> get(int warp, int slot, int g) const {
        const Head& h = head[warp][slot];
        UnitInfo<NB> u;
        u.pk = h.pk;
        u.sc = h.sc;
        u.zp = h.zp;
        u.ncols = h.ncols;
        u.tile = h.tile;
        u.split = h.split;
        u.unit = h.unit;
        u.ok = h.ok;
#pragma unroll
        for (int cb = 0; cb < NB; ++cb) u.col_row[cb] = rows[warp][slot][cb * 8 + g];
        return u;
    }
};

template <int NB>
__device__ __forceinline__ UnitInfo<NB> load_unit(const PassEntry* passes, int pg, int tile, int g) {
    UnitInfo<NB> u;
    const PassEntry& pe = passes[pg];
    u.pk = reinterpret_cast<const int32_t*>(pe.pk);
    u.sc = reinterpret_cast<const void*>(pe.sc);
    u.zp = reinterpret_cast<const int32_t*>(pe.zp);
    u.ncols = pe.ncols;
    u.tile = tile;
    u.split = 0;
    u.unit = 0;
#pragma unroll
    for (int cb = 0; cb < NB; ++cb) {
        const int col = cb * 8 + g;
        u.col_row[cb] = col < u.ncols ? pe.rows[col] : -1;
    }
    u.ok = u.pk != nullptr && u.sc != nullptr && (reinterpret_cast<uintptr_t>(u.pk) & 15u) == 0;
    return u;
}

// Activation-dtype bits of one scale, duplicated into both halves of a pair register.
template <int ACT, int SC>
__device__ __forceinline__ uint32_t scale_pair(const void* base, int64_t idx) {
    uint32_t b;
    if constexpr (SC == ACT) {
        b = __ldg(reinterpret_cast<const unsigned short*>(base) + idx);
    } else {
        b = act_bits<ACT>(load_scale<SC>(base, idx));
    }
    return __byte_perm(b, 0, 0x1010);
}

template <int ACT, bool ZERO>
__device__ __forceinline__ uint32_t bias_pair(const int32_t* zp, int64_t idx, int nib) {
    if constexpr (ZERO) {
        const uint32_t zw = static_cast<uint32_t>(__ldg(zp + idx));
        return int4_bias_pair<ACT>((zw >> (4 * nib)) & 15u);
    } else {
        return int4_bias_pair<ACT>(8u);
    }
}

// One 16-byte chunk (4 words = 32 codes) of one row, dequantised to 4 x 4 activation pairs.
template <int ACT>
__device__ __forceinline__ void dequant_chunk(const uint4& w, uint32_t bias, uint32_t scale,
                                              uint32_t (&a)[4][4]) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            a[wi][j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(words[wi], j), bias), scale);
}

template <int ACT, int SC, bool ZERO, int NB, bool SPLIT>
__global__ void __launch_bounds__(kGuWarps * 32, NB <= 2 ? 2 : 1) gate_up_kernel(GateUpParams p) {
    extern __shared__ uint4 ring[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    uint4* my_ring = ring + warp * (kGuDepth * 4 * 32);
    __shared__ UnitQueue<NB, kGuDepth, kGuWarps> queue;

    grid_dependency_wait();
    grid_dependents_launch();

    const int n_live = p.counters[0];
    if (n_live <= 0) return;
    const int tiles = p.inter / kTileRows;
    const int S = SPLIT ? p.k_splits : 1;          // 2, 4 or 8 in the split variant
    const int total_units = p.unit_start[n_live] * tiles * S;
    const int gw = blockIdx.x * kGuWarps + warp, nw = gridDim.x * kGuWarps;
    if (gw >= total_units) return;
    const int my_units = (total_units - gw + nw - 1) / nw;
    const int spu = p.hidden / kStageK;            // stages of a whole unit
    const int sps = spu / S;                       // stages of one split
    const int wpr = p.hidden / 8;
    const int groups = p.hidden >> p.gs_shift;

    // unit u: split u % S of (pass, tile) = u / S; the S splits of a tile go to adjacent warps
    auto unit_at = [&](int i) {
        const int u = gw + i * nw;
        const int ut = u / S;
        const int pg = ut / tiles;
        UnitInfo<NB> r = load_unit<NB>(p.passes, pg, ut - pg * tiles, g);
        if constexpr (SPLIT) {
            r.split = u - ut * S;
            r.unit = ut;
        }
        return r;
    };

    // ── issue side: kGuDepth - 1 stages ahead of the consuming side ─────────────────────────
    int i_ui = 0, i_ks = 0, i_slot = 0, i_left = my_units * sps;
    UnitInfo<NB> i_nxt = unit_at(0);
    const int32_t* i_src_g = nullptr;
    const int32_t* i_src_u = nullptr;
    bool i_ok = false;
    auto issue = [&]() {
        if (i_left > 0) {
            if (i_ks == 0) {
                const UnitInfo<NB> cur = i_nxt;
                queue.put(warp, i_ui % kGuDepth, lane, g, cur);
                if (i_ui + 1 < my_units) i_nxt = unit_at(i_ui + 1);
                i_ok = cur.ok;
                const int64_t row_off = int64_t(cur.tile * kTileRows + g) * wpr + tig * 4 +
                                        (SPLIT ? cur.split * sps * 16 : 0);
                i_src_g = cur.pk + p.w_off[0] + row_off;
                i_src_u = cur.pk + p.w_off[1] + row_off;
            }
            if (i_ok) {
                uint4* dst = my_ring + i_slot * 128 + lane;
                cp_async16(dst, i_src_g);
                cp_async16(dst + 32, i_src_g + 8 * wpr);
                cp_async16(dst + 64, i_src_u);
                cp_async16(dst + 96, i_src_u + 8 * wpr);
            }
            i_src_g += 16;
            i_src_u += 16;
            if (++i_ks == sps) {
                i_ks = 0;
                ++i_ui;
            }
            --i_left;
        }
        cp_async_commit();
        if (++i_slot == kGuDepth) i_slot = 0;
    };
#pragma unroll
    for (int s = 0; s < kGuDepth - 1; ++s) issue();

    // ── consuming side ───────────────────────────────────────────────────────────────────
    float acc_g[NB][4], acc_u[NB][4];
#pragma unroll
    for (int cb = 0; cb < NB; ++cb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc_g[cb][i] = acc_u[cb][i] = 0.f;
    UnitInfo<NB> cu{};
    int c_ui = 0, c_ks = 0, c_slot = 0;
    int xoff[NB];
    int sidx[4];      // scale element index of rows g, g+8 of gate, up at this thread's K offset
    int zidx[2];      // zero word index (rows g and g+8 share a nibble position) of gate, up
    const int kfirst = tig * 32;
    for (int s = my_units * sps; s > 0; --s) {
        issue();
        if (c_ks == 0) {
            __syncwarp();
            cu = queue.get(warp, c_ui % kGuDepth, g);
            const int row = cu.tile * kTileRows + g;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                sidx[2 * m] = static_cast<int>(p.s_off[m]) + row * groups;
                sidx[2 * m + 1] = sidx[2 * m] + 8 * groups;
                zidx[m] = static_cast<int>(p.z_off[m]) + (row >> 3) * groups;
            }
#pragma unroll
            for (int cb = 0; cb < NB; ++cb)
                xoff[cb] = cu.col_row[cb] >= 0 ? (cu.col_row[cb] / p.top_k) * p.hidden + kfirst : -1;
            if (!cu.ok && lane == 0) atomicOr(p.counters + 2, 1);
        }
        cp_async_wait<kGuDepth - 1>();
        if (cu.ok) {
            const int kx = ((SPLIT ? cu.split * sps : 0) + c_ks) * kStageK;
            // the first token block's activations first: their L2 latency hides behind the
            // dequant work below (further blocks, rarely populated at decode sizes, load in line)
            uint4 xv0[4];
#pragma unroll
            for (int wi = 0; wi < 4; ++wi)
                xv0[wi] = xoff[0] >= 0 ? ld_nc_v4(p.x_perm + xoff[0] + kx + wi * 8) : make_uint4(0u, 0u, 0u, 0u);
            const uint4* st = my_ring + c_slot * 128 + lane;
            const uint4 wg0 = st[0], wg8 = st[32], wu0 = st[64], wu8 = st[96];
            const int grp = (kx + kfirst) >> p.gs_shift;
            const uint32_t sg0 = scale_pair<ACT, SC>(cu.sc, sidx[0] + grp);
            const uint32_t sg8 = scale_pair<ACT, SC>(cu.sc, sidx[1] + grp);
            const uint32_t su0 = scale_pair<ACT, SC>(cu.sc, sidx[2] + grp);
            const uint32_t su8 = scale_pair<ACT, SC>(cu.sc, sidx[3] + grp);
            const uint32_t bg0 = bias_pair<ACT, ZERO>(cu.zp, zidx[0] + grp, g);
            const uint32_t bg8 = bias_pair<ACT, ZERO>(cu.zp, zidx[0] + groups + grp, g);
            const uint32_t bu0 = bias_pair<ACT, ZERO>(cu.zp, zidx[1] + grp, g);
            const uint32_t bu8 = bias_pair<ACT, ZERO>(cu.zp, zidx[1] + groups + grp, g);
            // The stage's 128-term partial dots start from zero and join the running sums with
            // round-to-nearest fp32 adds: the tensor core's own accumulate truncates against the
            // accumulator's magnitude, so a long chain inside it drifts (biased) from the fp32 sum.
            float sg[NB][4], su[NB][4];
#pragma unroll
            for (int cb = 0; cb < NB; ++cb)
#pragma unroll
                for (int i = 0; i < 4; ++i) sg[cb][i] = su[cb][i] = 0.f;
            const uint32_t wgw0[4] = {wg0.x, wg0.y, wg0.z, wg0.w}, wgw8[4] = {wg8.x, wg8.y, wg8.z, wg8.w};
            const uint32_t wuw0[4] = {wu0.x, wu0.y, wu0.z, wu0.w}, wuw8[4] = {wu8.x, wu8.y, wu8.z, wu8.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                uint32_t ag0[4], ag8[4], au0[4], au8[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    ag0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wgw0[wi], j), bg0), sg0);
                    ag8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wgw8[wi], j), bg8), sg8);
                    au0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wuw0[wi], j), bu0), su0);
                    au8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wuw8[wi], j), bu8), su8);
                }
#pragma unroll
                for (int cb = 0; cb < NB; ++cb) {
                    if (cb > 0 && cb * 8 >= cu.ncols) break;   // warp-uniform: no tokens left (a pass has one)
                    uint4 xv = xv0[wi];
                    if (cb > 0)
                        xv = xoff[cb] >= 0 ? ld_nc_v4(p.x_perm + xoff[cb] + kx + wi * 8) : make_uint4(0u, 0u, 0u, 0u);
                    mma_16816<ACT>(sg[cb], ag0[0], ag8[0], ag0[1], ag8[1], xv.x, xv.y);
                    mma_16816<ACT>(sg[cb], ag0[2], ag8[2], ag0[3], ag8[3], xv.z, xv.w);
                    mma_16816<ACT>(su[cb], au0[0], au8[0], au0[1], au8[1], xv.x, xv.y);
                    mma_16816<ACT>(su[cb], au0[2], au8[2], au0[3], au8[3], xv.z, xv.w);
                }
            }
            if constexpr (!SPLIT) {
#pragma unroll
                for (int cb = 0; cb < NB; ++cb) {
                    if (cb > 0 && cb * 8 >= cu.ncols) break;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        acc_g[cb][i] = __fadd_rn(acc_g[cb][i], sg[cb][i]);
                        acc_u[cb][i] = __fadd_rn(acc_u[cb][i], su[cb][i]);
                    }
                }
            } else {
                // split K: the stage's partial dots go to the unit's record, joined in stage order
                // by whichever split finishes last
                float4* rec = reinterpret_cast<float4*>(p.partial) +
                              ((int64_t(cu.unit) * spu + cu.split * sps + c_ks) * 32 + lane) * (2 * NB);
#pragma unroll
                for (int cb = 0; cb < NB; ++cb) {
                    if (cb > 0 && cb * 8 >= cu.ncols) break;
                    __stcg(rec + 2 * cb, make_float4(sg[cb][0], sg[cb][1], sg[cb][2], sg[cb][3]));
                    __stcg(rec + 2 * cb + 1, make_float4(su[cb][0], su[cb][1], su[cb][2], su[cb][3]));
                }
            }
        }
        if (++c_slot == kGuDepth) c_slot = 0;
        if (++c_ks == sps) {
            bool finish = true;
            if constexpr (SPLIT) {
                // publish this split's stages; the last split to arrive sums all of them in stage
                // order -- the same fp32 adds, in the same order, as one warp walking the unit
                __threadfence();
                __syncwarp();
                int prev = 0;
                if (lane == 0) prev = atomicAdd(p.tickets + cu.unit, 1);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                finish = prev == S - 1;
                if (finish && cu.ok) {
                    __threadfence();
                    const float4* rec = reinterpret_cast<const float4*>(p.partial) +
                                        (int64_t(cu.unit) * spu * 32 + lane) * (2 * NB);
                    for (int st = 0; st < spu; ++st) {
#pragma unroll
                        for (int cb = 0; cb < NB; ++cb) {
                            if (cb > 0 && cb * 8 >= cu.ncols) break;
                            const float4 a = __ldcg(rec + int64_t(st) * 32 * 2 * NB + 2 * cb);
                            const float4 b = __ldcg(rec + int64_t(st) * 32 * 2 * NB + 2 * cb + 1);
                            acc_g[cb][0] = __fadd_rn(acc_g[cb][0], a.x);
                            acc_g[cb][1] = __fadd_rn(acc_g[cb][1], a.y);
                            acc_g[cb][2] = __fadd_rn(acc_g[cb][2], a.z);
                            acc_g[cb][3] = __fadd_rn(acc_g[cb][3], a.w);
                            acc_u[cb][0] = __fadd_rn(acc_u[cb][0], b.x);
                            acc_u[cb][1] = __fadd_rn(acc_u[cb][1], b.y);
                            acc_u[cb][2] = __fadd_rn(acc_u[cb][2], b.z);
                            acc_u[cb][3] = __fadd_rn(acc_u[cb][3], b.w);
                        }
                    }
                }
            }
            if (finish && cu.ok) {
#pragma unroll
                for (int cb = 0; cb < NB; ++cb) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int col = cb * 8 + 2 * tig + (i & 1);
                        // every lane takes part in the shuffle; only live columns store
                        const int rowid = __shfl_sync(0xffffffffu, cu.col_row[cb], (col - cb * 8) * 4);
                        if (col < cu.ncols) {
                            const int r = cu.tile * kTileRows + g + 8 * (i >> 1);
                            const float gv = round_act<ACT>(acc_g[cb][i]);
                            const float uv = round_act<ACT>(acc_u[cb][i]);
                            const float av = round_act<ACT>(gv / (1.0f + expf(-gv)));
                            const uint32_t hb = act_bits<ACT>(__fmul_rn(av, uv));
                            p.h_perm[int64_t(rowid) * p.inter + perm8(r)] = static_cast<uint16_t>(hb);
                            if (p.h_out) p.h_out[int64_t(rowid) * p.inter + r] = static_cast<uint16_t>(hb);
                        }
                    }
                }
            }
#pragma unroll
            for (int cb = 0; cb < NB; ++cb)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc_g[cb][i] = acc_u[cb][i] = 0.f;
            c_ks = 0;
            ++c_ui;
        }
    }
    cp_async_wait<0>();
}

// The down projection, pass-major like gate/up: unit u = (pass u / tiles, 16-row tile u % tiles)
// dealt round-robin over every warp of one resident wave, so the eight warps of a CTA work on
// the same pass (the same h rows, shared through L1) and no warp has more than one unit above
// the average.  Each unit writes its 16 rows x (up to NB*8) weighted contributions to
// ybuf_g[row id][hidden]; the slot-ordered combine (or the expert-parallel caller) sums them.
template <int ACT, int SC, bool ZERO, int NB>
__global__ void __launch_bounds__(kWarps * 32, kDnBlocksPerSm[NB]) down_kernel(DownParams p) {
    extern __shared__ uint4 ring[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    uint4* my_ring = ring + warp * (kDnDepth * 2 * 32);
    __shared__ UnitQueue<NB, kDnDepth> queue;

    grid_dependency_wait();
    grid_dependents_launch();   // the combine may be scheduled now; it waits for this grid

    const int n_live = p.counters[0];
    if (n_live <= 0) return;
    const int tiles = p.hidden / kTileRows;
    const int total_units = p.unit_start[n_live] * tiles;
    const int gw = blockIdx.x * kWarps + warp, nw = gridDim.x * kWarps;
    if (gw >= total_units) return;
    const int my_units = (total_units - gw + nw - 1) / nw;
    const int spu = p.inter / kStageK;
    const int wpr = p.inter / 8;
    const int groups = p.inter >> p.gs_shift;
    auto unit_at = [&](int i) {
        const int u = gw + i * nw;
        const int pg = u / tiles;
        return load_unit<NB>(p.passes, pg, u - pg * tiles, g);
    };

    // ── issue side: kDnDepth - 1 stages ahead of the consuming side ─────────────────────────
    int i_ui = 0, i_ks = 0, i_slot = 0, i_left = my_units * spu;
    UnitInfo<NB> i_nxt = unit_at(0);
    const int32_t* i_src = nullptr;
    bool i_ok = false;
    auto issue = [&]() {
        if (i_left > 0) {
            if (i_ks == 0) {
                const UnitInfo<NB> cur = i_nxt;
                queue.put(warp, i_ui % kDnDepth, lane, g, cur);
                if (i_ui + 1 < my_units) i_nxt = unit_at(i_ui + 1);
                i_ok = cur.ok;
                i_src = cur.pk + p.w_off + int64_t(cur.tile * kTileRows + g) * wpr + tig * 4;
            }
            if (i_ok) {
                uint4* dst = my_ring + i_slot * 64 + lane;
                cp_async16(dst, i_src);
                cp_async16(dst + 32, i_src + 8 * wpr);
            }
            i_src += 16;
            if (++i_ks == spu) {
                i_ks = 0;
                ++i_ui;
            }
            --i_left;
        }
        cp_async_commit();
        if (++i_slot == kDnDepth) i_slot = 0;
    };
#pragma unroll
    for (int s = 0; s < kDnDepth - 1; ++s) issue();

    // ── consuming side ───────────────────────────────────────────────────────────────────
    float acc[NB][4];
#pragma unroll
    for (int cb = 0; cb < NB; ++cb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[cb][i] = 0.f;
    UnitInfo<NB> cu{};
    int c_ui = 0, c_ks = 0, c_slot = 0;
    int hoff[NB];
    int sidx0 = 0, zidx = 0;
    const int kfirst = tig * 32;
    for (int s = my_units * spu; s > 0; --s) {
        issue();
        if (c_ks == 0) {
            __syncwarp();
            cu = queue.get(warp, c_ui % kDnDepth, g);
            const int row = cu.tile * kTileRows + g;
            sidx0 = static_cast<int>(p.s_off) + row * groups;
            zidx = static_cast<int>(p.z_off) + (row >> 3) * groups;
#pragma unroll
            for (int cb = 0; cb < NB; ++cb)
                hoff[cb] = cu.col_row[cb] >= 0 ? cu.col_row[cb] * p.inter + kfirst : -1;
            if (!cu.ok && lane == 0) atomicOr(p.counters + 2, 1);
        }
        cp_async_wait<kDnDepth - 1>();
        if (cu.ok) {
            const int kh = c_ks * kStageK;
            uint4 hv0[4];
#pragma unroll
            for (int wi = 0; wi < 4; ++wi)
                hv0[wi] = hoff[0] >= 0 ? ld_nc_v4(p.h_perm + hoff[0] + kh + wi * 8) : make_uint4(0u, 0u, 0u, 0u);
            const uint4* st = my_ring + c_slot * 64 + lane;
            const uint4 w0 = st[0], w8 = st[32];
            const int grp = (kh + kfirst) >> p.gs_shift;
            const uint32_t s0 = scale_pair<ACT, SC>(cu.sc, sidx0 + grp);
            const uint32_t s8 = scale_pair<ACT, SC>(cu.sc, sidx0 + 8 * groups + grp);
            const uint32_t b0 = bias_pair<ACT, ZERO>(cu.zp, zidx + grp, g);
            const uint32_t b8 = bias_pair<ACT, ZERO>(cu.zp, zidx + groups + grp, g);
            float sp[NB][4];   // the stage's partial dots (see gate_up_kernel)
#pragma unroll
            for (int cb = 0; cb < NB; ++cb)
#pragma unroll
                for (int i = 0; i < 4; ++i) sp[cb][i] = 0.f;
            const uint32_t ww0[4] = {w0.x, w0.y, w0.z, w0.w}, ww8[4] = {w8.x, w8.y, w8.z, w8.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                uint32_t a0[4], a8[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    a0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(ww0[wi], j), b0), s0);
                    a8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(ww8[wi], j), b8), s8);
                }
#pragma unroll
                for (int cb = 0; cb < NB; ++cb) {
                    if (cb > 0 && cb * 8 >= cu.ncols) break;   // warp-uniform: no tokens left (a pass has one)
                    uint4 hv = hv0[wi];
                    if (cb > 0)
                        hv = hoff[cb] >= 0 ? ld_nc_v4(p.h_perm + hoff[cb] + kh + wi * 8) : make_uint4(0u, 0u, 0u, 0u);
                    mma_16816<ACT>(sp[cb], a0[0], a8[0], a0[1], a8[1], hv.x, hv.y);
                    mma_16816<ACT>(sp[cb], a0[2], a8[2], a0[3], a8[3], hv.z, hv.w);
                }
            }
#pragma unroll
            for (int cb = 0; cb < NB; ++cb) {
                if (cb > 0 && cb * 8 >= cu.ncols) break;
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[cb][i] = __fadd_rn(acc[cb][i], sp[cb][i]);
            }
        }
        if (++c_slot == kDnDepth) c_slot = 0;
        if (++c_ks == spu) {
            if (cu.ok) {
#pragma unroll
                for (int cb = 0; cb < NB; ++cb) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int col = cb * 8 + 2 * tig + (i & 1);
                        const int rowid = __shfl_sync(0xffffffffu, cu.col_row[cb], (col - cb * 8) * 4);
                        if (col < cu.ncols) {
                            const int r = cu.tile * kTileRows + g + 8 * (i >> 1);
                            const int64_t t = rowid / p.top_k;
                            const int k = rowid - int(t) * p.top_k;
                            const int widx = p.w_index ? p.w_index[rowid] : k;
                            const float wv = load_as_float(p.weights, p.w_dtype,
                                                           t * p.w_tok_stride + int64_t(widx) * p.w_slot_stride);
                            float c = __fmul_rn(round_act<ACT>(acc[cb][i]), wv);
                            if (p.w_round) c = round_act<ACT>(c);
                            p.ybuf_g[int64_t(rowid) * p.hidden + r] = c;
                        }
                    }
                }
            }
#pragma unroll
            for (int cb = 0; cb < NB; ++cb)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[cb][i] = 0.f;
            c_ks = 0;
            ++c_ui;
        }
    }
    cp_async_wait<0>();
}

// ── few-row calls: one CTA per (routed row, 16-row tile), no routing plan ────────────────
//
// A call of at most kRowMaxRows routed rows (a token or two at top-8) is latency-bound: the plan
// kernel, the persistent grids' unit hand-off and the split-K join through global memory cost
// more than moving its weights.  Here every CTA looks up its own row's expert, its warps share
// the tile's K range (contiguous stage ranges, each streamed through a small cp.async ring), and
// the stages' partial dots meet in shared memory, summed in stage order by one thread per output
// row.  The per-stage MMA chains and that stage-order sum are the ones gate_up_kernel and
// down_kernel perform, so the result is bit-identical to the planned path's.  A row routed to an
// expert outside the table (or to one whose streams are unusable) contributes zero; the
// layer's combine then sums each token's slots in ascending expert id, then slot.

#ifndef VY_ROW_GU_WARPS
#define VY_ROW_GU_WARPS 8
#endif
#ifndef VY_ROW_DN_WARPS
#define VY_ROW_DN_WARPS 4
#endif
#ifndef VY_ROW_DEPTH
#define VY_ROW_DEPTH 3
#endif
constexpr int kRowMaxRows = 16;
constexpr int kRowGuWarps = VY_ROW_GU_WARPS;   // warps sharing a gate/up tile's K range
constexpr int kRowDnWarps = VY_ROW_DN_WARPS;   // warps sharing a down tile's K range
constexpr int kRowDepth = VY_ROW_DEPTH;        // ring stages per warp (kRowDepth - 1 in flight)
constexpr int kRowMaxStages = 64;     // hidden / 128 and intermediate / 128 (stash bound)

struct RowParams {
    const void* ids;
    bool ids64;
    int64_t ids_stride;
    int id_base, n_experts, top_k, n_rows;
    const int64_t* table;
    int hidden, inter, gs_shift;
    int64_t w_off[3], s_off[3], z_off[3];   // gate, up, down
    const void* x;
    int64_t x_stride;
    bool x_vec;
    uint16_t* h_perm;
    uint16_t* h_out;
    const void* weights;
    int w_dtype;
    bool w_round;
    int64_t w_tok_stride, w_slot_stride;
    const int32_t* w_index;
    float* contrib;       // [n_rows][hidden] weighted contributions, by row id
    int32_t* flags;       // the call's error flags (one word)
    float* out;           // the layer's combine into out [n_tokens, out_stride] (null: contributions only)
    int64_t out_stride;
    int32_t* tickets;     // [n_tokens][hidden / 16], zeroed by the gate/up kernel
};

__device__ __forceinline__ int row_id_load(const void* ids, bool ids64, int64_t j) {
    if (ids64) {
        const int64_t v = reinterpret_cast<const int64_t*>(ids)[j];
        return (v < INT32_MIN || v > INT32_MAX) ? -1 : static_cast<int>(v);
    }
    return reinterpret_cast<const int32_t*>(ids)[j];
}

struct RowExpert {
    const int32_t* pk;
    const void* sc;
    const int32_t* zp;
    bool ok;              // routed to this table and its streams usable
    bool bad;             // routed to this table but its streams unusable
};

__device__ __forceinline__ RowExpert row_expert(const RowParams& p, int r) {
    const int64_t t = r / p.top_k;
    int e = row_id_load(p.ids, p.ids64, t * p.ids_stride + (r - t * p.top_k));
    e = (e < 0) ? -1 : e - p.id_base;
    RowExpert x{nullptr, nullptr, nullptr, false, false};
    if (e < 0 || e >= p.n_experts) return x;
    x.pk = reinterpret_cast<const int32_t*>(p.table[3 * int64_t(e)]);
    x.sc = reinterpret_cast<const void*>(p.table[3 * int64_t(e) + 1]);
    x.zp = reinterpret_cast<const int32_t*>(p.table[3 * int64_t(e) + 2]);
    x.ok = x.pk != nullptr && x.sc != nullptr && (reinterpret_cast<uintptr_t>(x.pk) & 15u) == 0;
    x.bad = !x.ok;
    return x;
}

// One warp's share of a tile's K range: stages [lo, hi) of `spu`, through a DEPTH-stage ring of
// `chunks` 16-byte copies per lane and stage.  `src(stage, c)` is copy c's global address.
template <int CHUNKS, int DEPTH, typename Src>
struct RowRing {
    uint4* ring;          // this warp's [DEPTH][CHUNKS][32]
    int lo, hi, next;
    __device__ __forceinline__ void issue(const Src& src, int lane) {
        if (next < hi) {
            uint4* dst = ring + ((next - lo) % DEPTH) * (CHUNKS * 32) + lane;
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c) cp_async16(dst + 32 * c, src(next, c));
        }
        cp_async_commit();
        ++next;
    }
    __device__ __forceinline__ const uint4* slot(int stage, int lane) const {
        return ring + ((stage - lo) % DEPTH) * (CHUNKS * 32) + lane;
    }
};

// After a down CTA has stored its 16 contributions of row r: the last of token t's top_k rows to
// finish this 16-column tile sums them into `out`, in ascending expert id, then slot (ids below
// zero skipped) -- the order of the layer's combine, whichever CTA arrives last.
__device__ __forceinline__ void row_combine(const RowParams& p, int r, int tile) {
    if (!p.out) return;
    __shared__ int last;
    const int64_t t = r / p.top_k;
    if (threadIdx.x < kTileRows) __threadfence();      // this thread's contribution is visible
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(p.tickets + t * (p.hidden / kTileRows) + tile, 1);
        last = prev == p.top_k - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x >= kTileRows) return;
    __threadfence();
    int key[kMaxTopK], idx[kMaxTopK];
    for (int k = 0; k < p.top_k; ++k) {
        const int e = row_id_load(p.ids, p.ids64, t * p.ids_stride + k);
        key[k] = e < 0 ? INT32_MAX : e;
        idx[k] = k;
    }
    for (int a = 1; a < p.top_k; ++a) {
        const int kv = key[a], iv = idx[a];
        int b = a - 1;
        while (b >= 0 && key[b] > kv) {
            key[b + 1] = key[b];
            idx[b + 1] = idx[b];
            --b;
        }
        key[b + 1] = kv;
        idx[b + 1] = iv;
    }
    const int64_t col = int64_t(tile) * kTileRows + threadIdx.x;
    float acc = 0.f;
    for (int k = 0; k < p.top_k; ++k)
        if (key[k] != INT32_MAX) acc += __ldcg(p.contrib + (t * p.top_k + idx[k]) * p.hidden + col);
    p.out[t * p.out_stride + col] = acc;
}

template <int ACT, int SC, bool ZERO>
__global__ void __launch_bounds__(kRowGuWarps * 32) row_gate_up_kernel(RowParams p) {
    extern __shared__ uint4 row_smem[];   // rings [kRowGuWarps][kRowDepth][4][32], then x (permuted)
    __shared__ float stash[kRowMaxStages][kTileRows][2];
    grid_dependency_wait();
    grid_dependents_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const int tile = blockIdx.x, r = blockIdx.y;
    if (tile == 0 && r == 0) {
        // the call's error flags, written whole: a routed expert's streams unusable
        if (threadIdx.x == 0) {
            int32_t f = 0;
            for (int q = 0; q < p.n_rows; ++q) f |= row_expert(p, q).bad ? 1 : 0;
            *p.flags = f;
        }
        // the down kernel's combine tickets (it runs after this grid has completed)
        if (p.out)
            for (int i = threadIdx.x; i < (p.n_rows / p.top_k) * (p.hidden / kTileRows); i += blockDim.x)
                p.tickets[i] = 0;
    }
    const RowExpert ex = row_expert(p, r);
    if (!ex.ok) return;                   // no h row: the down kernel gives this row zeros
    const int64_t t = r / p.top_k;
    // this token's activations in the pair-permuted order (code j, code j + 4) of int4_pair
    uint16_t* xs = reinterpret_cast<uint16_t*>(row_smem + kRowGuWarps * kRowDepth * 4 * 32);
    const uint16_t* xt = reinterpret_cast<const uint16_t*>(p.x) + t * p.x_stride;
    for (int c8 = threadIdx.x; c8 < p.hidden / 8; c8 += blockDim.x) {
        uint16_t v[8];
        if (p.x_vec) {
            *reinterpret_cast<uint4*>(v) = *reinterpret_cast<const uint4*>(xt + c8 * 8);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = xt[c8 * 8 + j];
        }
        uint4 o;
        o.x = v[0] | (uint32_t(v[4]) << 16);
        o.y = v[1] | (uint32_t(v[5]) << 16);
        o.z = v[2] | (uint32_t(v[6]) << 16);
        o.w = v[3] | (uint32_t(v[7]) << 16);
        *reinterpret_cast<uint4*>(xs + c8 * 8) = o;
    }
    const int spu = p.hidden / kStageK, wpr = p.hidden / 8, groups = p.hidden >> p.gs_shift;
    const int row = tile * kTileRows + g;
    const int32_t* srcg = ex.pk + p.w_off[0] + int64_t(row) * wpr + tig * 4;
    const int32_t* srcu = ex.pk + p.w_off[1] + int64_t(row) * wpr + tig * 4;
    auto src = [&](int stage, int c) -> const int32_t* {
        const int32_t* b = (c < 2 ? srcg : srcu) + stage * 16;
        return (c & 1) ? b + 8 * wpr : b;
    };
    RowRing<4, kRowDepth, decltype(src)> rg{row_smem + warp * (kRowDepth * 4 * 32), warp * spu / kRowGuWarps,
                                 (warp + 1) * spu / kRowGuWarps, warp * spu / kRowGuWarps};
#pragma unroll
    for (int d = 0; d < kRowDepth - 1; ++d) rg.issue(src, lane);
    __syncthreads();                      // xs complete
    int sidx[4], zidx[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        sidx[2 * m] = static_cast<int>(p.s_off[m]) + row * groups;
        sidx[2 * m + 1] = sidx[2 * m] + 8 * groups;
        zidx[m] = static_cast<int>(p.z_off[m]) + (row >> 3) * groups;
    }
    const int kfirst = tig * 32;
    for (int st = rg.lo; st < rg.hi; ++st) {
        rg.issue(src, lane);
        cp_async_wait<kRowDepth - 1>();
        const int kx = st * kStageK;
        uint4 xv[4];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) xv[wi] = *reinterpret_cast<const uint4*>(xs + kx + kfirst + wi * 8);
        const uint4* sl = rg.slot(st, lane);
        const uint4 wg0 = sl[0], wg8 = sl[32], wu0 = sl[64], wu8 = sl[96];
        const int grp = (kx + kfirst) >> p.gs_shift;
        const uint32_t sg0 = scale_pair<ACT, SC>(ex.sc, sidx[0] + grp);
        const uint32_t sg8 = scale_pair<ACT, SC>(ex.sc, sidx[1] + grp);
        const uint32_t su0 = scale_pair<ACT, SC>(ex.sc, sidx[2] + grp);
        const uint32_t su8 = scale_pair<ACT, SC>(ex.sc, sidx[3] + grp);
        const uint32_t bg0 = bias_pair<ACT, ZERO>(ex.zp, zidx[0] + grp, g);
        const uint32_t bg8 = bias_pair<ACT, ZERO>(ex.zp, zidx[0] + groups + grp, g);
        const uint32_t bu0 = bias_pair<ACT, ZERO>(ex.zp, zidx[1] + grp, g);
        const uint32_t bu8 = bias_pair<ACT, ZERO>(ex.zp, zidx[1] + groups + grp, g);
        float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t wgw0[4] = {wg0.x, wg0.y, wg0.z, wg0.w}, wgw8[4] = {wg8.x, wg8.y, wg8.z, wg8.w};
        const uint32_t wuw0[4] = {wu0.x, wu0.y, wu0.z, wu0.w}, wuw8[4] = {wu8.x, wu8.y, wu8.z, wu8.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            uint32_t ag0[4], ag8[4], au0[4], au8[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                ag0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wgw0[wi], j), bg0), sg0);
                ag8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wgw8[wi], j), bg8), sg8);
                au0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wuw0[wi], j), bu0), su0);
                au8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wuw8[wi], j), bu8), su8);
            }
            mma_16816<ACT>(sg, ag0[0], ag8[0], ag0[1], ag8[1], xv[wi].x, xv[wi].y);
            mma_16816<ACT>(sg, ag0[2], ag8[2], ag0[3], ag8[3], xv[wi].z, xv[wi].w);
            mma_16816<ACT>(su, au0[0], au8[0], au0[1], au8[1], xv[wi].x, xv[wi].y);
            mma_16816<ACT>(su, au0[2], au8[2], au0[3], au8[3], xv[wi].z, xv[wi].w);
        }
        if (tig == 0) {                   // column 0 of the fragment is the token
            stash[st][g][0] = sg[0];
            stash[st][g + 8][0] = sg[2];
            stash[st][g][1] = su[0];
            stash[st][g + 8][1] = su[2];
        }
    }
    cp_async_wait<0>();
    __syncthreads();
    if (threadIdx.x < kTileRows) {
        const int rr = threadIdx.x;
        float ag = 0.f, au = 0.f;
        for (int st = 0; st < spu; ++st) {
            ag = __fadd_rn(ag, stash[st][rr][0]);
            au = __fadd_rn(au, stash[st][rr][1]);
        }
        const int rrow = tile * kTileRows + rr;
        const float gv = round_act<ACT>(ag);
        const float uv = round_act<ACT>(au);
        const float av = round_act<ACT>(gv / (1.0f + expf(-gv)));
        const uint32_t hb = act_bits<ACT>(__fmul_rn(av, uv));
        p.h_perm[int64_t(r) * p.inter + perm8(rrow)] = static_cast<uint16_t>(hb);
        if (p.h_out) p.h_out[int64_t(r) * p.inter + rrow] = static_cast<uint16_t>(hb);
    }
}

template <int ACT, int SC, bool ZERO>
__global__ void __launch_bounds__(kRowDnWarps * 32) row_down_kernel(RowParams p) {
    extern __shared__ uint4 row_smem[];   // rings [kRowDnWarps][kRowDepth][2][32]
    __shared__ float stash[kRowMaxStages][kTileRows];
    // Launched chained to the gate/up grid, which starts after the call's inputs are complete: the
    // routing ids and the expert table may be read, and this row's down weights fetched, while
    // that grid still runs; h and the combine tickets only after it has finished.
    grid_dependents_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const int tile = blockIdx.x, r = blockIdx.y;
    const RowExpert ex = row_expert(p, r);
    if (!ex.ok) {                         // not this table's row: it adds nothing to the combine
        grid_dependency_wait();
        if (threadIdx.x < kTileRows) p.contrib[int64_t(r) * p.hidden + tile * kTileRows + threadIdx.x] = 0.f;
        row_combine(p, r, tile);
        return;
    }
    const int spu = p.inter / kStageK, wpr = p.inter / 8, groups = p.inter >> p.gs_shift;
    const int row = tile * kTileRows + g;
    const int32_t* srcd = ex.pk + p.w_off[2] + int64_t(row) * wpr + tig * 4;
    auto src = [&](int stage, int c) -> const int32_t* { return srcd + stage * 16 + (c ? 8 * wpr : 0); };
    RowRing<2, kRowDepth, decltype(src)> rg{row_smem + warp * (kRowDepth * 2 * 32), warp * spu / kRowDnWarps,
                                 (warp + 1) * spu / kRowDnWarps, warp * spu / kRowDnWarps};
#pragma unroll
    for (int d = 0; d < kRowDepth - 1; ++d) rg.issue(src, lane);
    grid_dependency_wait();
    const int sidx0 = static_cast<int>(p.s_off[2]) + row * groups;
    const int zidx = static_cast<int>(p.z_off[2]) + (row >> 3) * groups;
    const int kfirst = tig * 32;
    const uint16_t* hrow = p.h_perm + int64_t(r) * p.inter + kfirst;
    for (int st = rg.lo; st < rg.hi; ++st) {
        rg.issue(src, lane);
        const int kh = st * kStageK;
        uint4 hv[4];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) hv[wi] = ld_nc_v4(hrow + kh + wi * 8);
        cp_async_wait<kRowDepth - 1>();
        const uint4* sl = rg.slot(st, lane);
        const uint4 w0 = sl[0], w8 = sl[32];
        const int grp = (kh + kfirst) >> p.gs_shift;
        const uint32_t s0 = scale_pair<ACT, SC>(ex.sc, sidx0 + grp);
        const uint32_t s8 = scale_pair<ACT, SC>(ex.sc, sidx0 + 8 * groups + grp);
        const uint32_t b0 = bias_pair<ACT, ZERO>(ex.zp, zidx + grp, g);
        const uint32_t b8 = bias_pair<ACT, ZERO>(ex.zp, zidx + groups + grp, g);
        float sp[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t ww0[4] = {w0.x, w0.y, w0.z, w0.w}, ww8[4] = {w8.x, w8.y, w8.z, w8.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            uint32_t a0[4], a8[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                a0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(ww0[wi], j), b0), s0);
                a8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(ww8[wi], j), b8), s8);
            }
            mma_16816<ACT>(sp, a0[0], a8[0], a0[1], a8[1], hv[wi].x, hv[wi].y);
            mma_16816<ACT>(sp, a0[2], a8[2], a0[3], a8[3], hv[wi].z, hv[wi].w);
        }
        if (tig == 0) {
            stash[st][g] = sp[0];
            stash[st][g + 8] = sp[2];
        }
    }
    cp_async_wait<0>();
    __syncthreads();
    if (threadIdx.x < kTileRows) {
        const int rr = threadIdx.x;
        float acc = 0.f;
        for (int st = 0; st < spu; ++st) acc = __fadd_rn(acc, stash[st][rr]);
        const int64_t t = r / p.top_k;
        const int k = r - int(t) * p.top_k;
        const int widx = p.w_index ? p.w_index[r] : k;
        const float wv = load_as_float(p.weights, p.w_dtype, t * p.w_tok_stride + int64_t(widx) * p.w_slot_stride);
        float c = __fmul_rn(round_act<ACT>(acc), wv);
        if (p.w_round) c = round_act<ACT>(c);
        p.contrib[int64_t(r) * p.hidden + tile * kTileRows + rr] = c;
    }
    row_combine(p, r, tile);
}

// ── planned calls, one CTA per (pass, 16-row tile) ─────────────────────────────────────
//
// The same units as gate_up_kernel / down_kernel (a pass of a live expert: up to 8 routed rows;
// a 16-row tile), but a unit is a CTA whose warps share its K range, instead of a warp walking the
// whole K range: more loads in flight per unit and no per-warp unit hand-off.  The stage partials
// of every column meet in shared memory and are added in stage order, so the results are
// bit-identical to the warp-unit kernels'.  The grid covers the largest possible pass count; CTAs
// past the call's passes exit at once.

#ifndef VY_PASS_GU_WARPS
#define VY_PASS_GU_WARPS 8
#endif
#ifndef VY_PASS_DN_WARPS
#define VY_PASS_DN_WARPS 4
#endif
#ifndef VY_PASS_DEPTH
#define VY_PASS_DEPTH 2
#endif
constexpr int kPassGuWarps = VY_PASS_GU_WARPS;
constexpr int kPassDnWarps = VY_PASS_DN_WARPS;
constexpr int kPassDepth = VY_PASS_DEPTH;     // ring stages per warp (one in flight ahead)
constexpr int kPassMaxRows = 64;              // routed rows a call may have to take these kernels

size_t pass_gu_smem(int hidden) {
    return size_t(kPassGuWarps) * kPassDepth * 4 * 32 * sizeof(uint4) + size_t(hidden / kStageK) * kTileRows * 2 * 8 * 4;
}
size_t pass_dn_smem(int inter) {
    return size_t(kPassDnWarps) * kPassDepth * 2 * 32 * sizeof(uint4) + size_t(inter / kStageK) * kTileRows * 8 * 4;
}

template <int ACT, int SC, bool ZERO>
__global__ void __launch_bounds__(kPassGuWarps * 32) pass_gate_up_kernel(GateUpParams p) {
    extern __shared__ uint4 pass_smem[];  // rings [kPassGuWarps][kPassDepth][4][32], then the stash
    __shared__ int col_row[8];
    __shared__ int ncols_s;
    grid_dependency_wait();
    grid_dependents_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const int tile = blockIdx.x, pg = blockIdx.y;
    const int n_live = p.counters[0];
    if (n_live <= 0 || pg >= p.unit_start[n_live]) return;
    const PassEntry& pe = p.passes[pg];
    const int32_t* pk = reinterpret_cast<const int32_t*>(pe.pk);
    const void* sc = reinterpret_cast<const void*>(pe.sc);
    const int32_t* zp = reinterpret_cast<const int32_t*>(pe.zp);
    const bool ok = pk != nullptr && sc != nullptr && (reinterpret_cast<uintptr_t>(pk) & 15u) == 0;
    if (!ok) {
        if (tile == 0 && threadIdx.x == 0) atomicOr(p.counters + 2, 1);
        return;
    }
    if (threadIdx.x < 8) col_row[threadIdx.x] = threadIdx.x < pe.ncols ? pe.rows[threadIdx.x] : -1;
    if (threadIdx.x == 0) ncols_s = pe.ncols < 8 ? pe.ncols : 8;
    const int spu = p.hidden / kStageK, wpr = p.hidden / 8, groups = p.hidden >> p.gs_shift;
    const int row = tile * kTileRows + g;
    const int32_t* srcg = pk + p.w_off[0] + int64_t(row) * wpr + tig * 4;
    const int32_t* srcu = pk + p.w_off[1] + int64_t(row) * wpr + tig * 4;
    auto src = [&](int stage, int c) -> const int32_t* {
        const int32_t* b = (c < 2 ? srcg : srcu) + stage * 16;
        return (c & 1) ? b + 8 * wpr : b;
    };
    RowRing<4, kPassDepth, decltype(src)> rg{pass_smem + warp * (kPassDepth * 4 * 32), warp * spu / kPassGuWarps,
                                 (warp + 1) * spu / kPassGuWarps, warp * spu / kPassGuWarps};
#pragma unroll
    for (int d = 0; d < kPassDepth - 1; ++d) rg.issue(src, lane);
    float* stash = reinterpret_cast<float*>(pass_smem + kPassGuWarps * kPassDepth * 4 * 32);   // [spu][16][2][8]
    __syncthreads();                      // col_row
    const int myrow = col_row[g];         // this lane's column (token row) in the fragments
    const int kfirst = tig * 32;
    const int xoff = myrow >= 0 ? (myrow / p.top_k) * p.hidden + kfirst : -1;
    int sidx[4], zidx[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        sidx[2 * m] = static_cast<int>(p.s_off[m]) + row * groups;
        sidx[2 * m + 1] = sidx[2 * m] + 8 * groups;
        zidx[m] = static_cast<int>(p.z_off[m]) + (row >> 3) * groups;
    }
    for (int st = rg.lo; st < rg.hi; ++st) {
        rg.issue(src, lane);
        const int kx = st * kStageK;
        uint4 xv[4];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi)
            xv[wi] = xoff >= 0 ? ld_nc_v4(p.x_perm + xoff + kx + wi * 8) : make_uint4(0u, 0u, 0u, 0u);
        cp_async_wait<kPassDepth - 1>();
        const uint4* sl = rg.slot(st, lane);
        const uint4 wg0 = sl[0], wg8 = sl[32], wu0 = sl[64], wu8 = sl[96];
        const int grp = (kx + kfirst) >> p.gs_shift;
        const uint32_t sg0 = scale_pair<ACT, SC>(sc, sidx[0] + grp);
        const uint32_t sg8 = scale_pair<ACT, SC>(sc, sidx[1] + grp);
        const uint32_t su0 = scale_pair<ACT, SC>(sc, sidx[2] + grp);
        const uint32_t su8 = scale_pair<ACT, SC>(sc, sidx[3] + grp);
        const uint32_t bg0 = bias_pair<ACT, ZERO>(zp, zidx[0] + grp, g);
        const uint32_t bg8 = bias_pair<ACT, ZERO>(zp, zidx[0] + groups + grp, g);
        const uint32_t bu0 = bias_pair<ACT, ZERO>(zp, zidx[1] + grp, g);
        const uint32_t bu8 = bias_pair<ACT, ZERO>(zp, zidx[1] + groups + grp, g);
        float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t wgw0[4] = {wg0.x, wg0.y, wg0.z, wg0.w}, wgw8[4] = {wg8.x, wg8.y, wg8.z, wg8.w};
        const uint32_t wuw0[4] = {wu0.x, wu0.y, wu0.z, wu0.w}, wuw8[4] = {wu8.x, wu8.y, wu8.z, wu8.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            uint32_t ag0[4], ag8[4], au0[4], au8[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                ag0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wgw0[wi], j), bg0), sg0);
                ag8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wgw8[wi], j), bg8), sg8);
                au0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wuw0[wi], j), bu0), su0);
                au8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(wuw8[wi], j), bu8), su8);
            }
            mma_16816<ACT>(sg, ag0[0], ag8[0], ag0[1], ag8[1], xv[wi].x, xv[wi].y);
            mma_16816<ACT>(sg, ag0[2], ag8[2], ag0[3], ag8[3], xv[wi].z, xv[wi].w);
            mma_16816<ACT>(su, au0[0], au8[0], au0[1], au8[1], xv[wi].x, xv[wi].y);
            mma_16816<ACT>(su, au0[2], au8[2], au0[3], au8[3], xv[wi].z, xv[wi].w);
        }
        // fragment (row g / g + 8, columns 2 tig / 2 tig + 1) into the stash [st][row][g or u][col]
        float* sa = stash + ((st * kTileRows + g) * 2) * 8 + 2 * tig;
        float* sb = stash + ((st * kTileRows + g + 8) * 2) * 8 + 2 * tig;
        *reinterpret_cast<float2*>(sa) = make_float2(sg[0], sg[1]);
        *reinterpret_cast<float2*>(sa + 8) = make_float2(su[0], su[1]);
        *reinterpret_cast<float2*>(sb) = make_float2(sg[2], sg[3]);
        *reinterpret_cast<float2*>(sb + 8) = make_float2(su[2], su[3]);
    }
    cp_async_wait<0>();
    __syncthreads();
    if (threadIdx.x < kTileRows * 8) {
        const int rr = threadIdx.x >> 3, c = threadIdx.x & 7;
        if (c < ncols_s) {
            float ag = 0.f, au = 0.f;
            for (int st = 0; st < spu; ++st) {
                ag = __fadd_rn(ag, stash[((st * kTileRows + rr) * 2) * 8 + c]);
                au = __fadd_rn(au, stash[((st * kTileRows + rr) * 2 + 1) * 8 + c]);
            }
            const int rrow = tile * kTileRows + rr, rowid = col_row[c];
            const float gv = round_act<ACT>(ag);
            const float uv = round_act<ACT>(au);
            const float av = round_act<ACT>(gv / (1.0f + expf(-gv)));
            const uint32_t hb = act_bits<ACT>(__fmul_rn(av, uv));
            p.h_perm[int64_t(rowid) * p.inter + perm8(rrow)] = static_cast<uint16_t>(hb);
            if (p.h_out) p.h_out[int64_t(rowid) * p.inter + rrow] = static_cast<uint16_t>(hb);
        }
    }
}

template <int ACT, int SC, bool ZERO>
__global__ void __launch_bounds__(kPassDnWarps * 32) pass_down_kernel(DownParams p) {
    extern __shared__ uint4 pass_smem[];  // rings [kPassDnWarps][kPassDepth][2][32], then the stash
    __shared__ int col_row[8];
    __shared__ int ncols_s;
    grid_dependency_wait();
    grid_dependents_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const int tile = blockIdx.x, pg = blockIdx.y;
    const int n_live = p.counters[0];
    if (n_live <= 0 || pg >= p.unit_start[n_live]) return;
    const PassEntry& pe = p.passes[pg];
    const int32_t* pk = reinterpret_cast<const int32_t*>(pe.pk);
    const void* sc = reinterpret_cast<const void*>(pe.sc);
    const int32_t* zp = reinterpret_cast<const int32_t*>(pe.zp);
    const bool ok = pk != nullptr && sc != nullptr && (reinterpret_cast<uintptr_t>(pk) & 15u) == 0;
    if (!ok) return;                      // flagged by the gate/up kernel
    if (threadIdx.x < 8) col_row[threadIdx.x] = threadIdx.x < pe.ncols ? pe.rows[threadIdx.x] : -1;
    if (threadIdx.x == 0) ncols_s = pe.ncols < 8 ? pe.ncols : 8;
    const int spu = p.inter / kStageK, wpr = p.inter / 8, groups = p.inter >> p.gs_shift;
    const int row = tile * kTileRows + g;
    const int32_t* srcd = pk + p.w_off + int64_t(row) * wpr + tig * 4;
    auto src = [&](int stage, int c) -> const int32_t* { return srcd + stage * 16 + (c ? 8 * wpr : 0); };
    RowRing<2, kPassDepth, decltype(src)> rg{pass_smem + warp * (kPassDepth * 2 * 32), warp * spu / kPassDnWarps,
                                 (warp + 1) * spu / kPassDnWarps, warp * spu / kPassDnWarps};
#pragma unroll
    for (int d = 0; d < kPassDepth - 1; ++d) rg.issue(src, lane);
    float* stash = reinterpret_cast<float*>(pass_smem + kPassDnWarps * kPassDepth * 2 * 32);   // [spu][16][8]
    __syncthreads();
    const int myrow = col_row[g];
    const int kfirst = tig * 32;
    const int hoff = myrow >= 0 ? myrow * p.inter + kfirst : -1;
    const int sidx0 = static_cast<int>(p.s_off) + row * groups;
    const int zidx = static_cast<int>(p.z_off) + (row >> 3) * groups;
    for (int st = rg.lo; st < rg.hi; ++st) {
        rg.issue(src, lane);
        const int kh = st * kStageK;
        uint4 hv[4];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi)
            hv[wi] = hoff >= 0 ? ld_nc_v4(p.h_perm + hoff + kh + wi * 8) : make_uint4(0u, 0u, 0u, 0u);
        cp_async_wait<kPassDepth - 1>();
        const uint4* sl = rg.slot(st, lane);
        const uint4 w0 = sl[0], w8 = sl[32];
        const int grp = (kh + kfirst) >> p.gs_shift;
        const uint32_t s0 = scale_pair<ACT, SC>(sc, sidx0 + grp);
        const uint32_t s8 = scale_pair<ACT, SC>(sc, sidx0 + 8 * groups + grp);
        const uint32_t b0 = bias_pair<ACT, ZERO>(zp, zidx + grp, g);
        const uint32_t b8 = bias_pair<ACT, ZERO>(zp, zidx + groups + grp, g);
        float sp[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t ww0[4] = {w0.x, w0.y, w0.z, w0.w}, ww8[4] = {w8.x, w8.y, w8.z, w8.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            uint32_t a0[4], a8[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                a0[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(ww0[wi], j), b0), s0);
                a8[j] = pair_mul<ACT>(pair_sub<ACT>(int4_pair<ACT>(ww8[wi], j), b8), s8);
            }
            mma_16816<ACT>(sp, a0[0], a8[0], a0[1], a8[1], hv[wi].x, hv[wi].y);
            mma_16816<ACT>(sp, a0[2], a8[2], a0[3], a8[3], hv[wi].z, hv[wi].w);
        }
        *reinterpret_cast<float2*>(stash + (st * kTileRows + g) * 8 + 2 * tig) = make_float2(sp[0], sp[1]);
        *reinterpret_cast<float2*>(stash + (st * kTileRows + g + 8) * 8 + 2 * tig) = make_float2(sp[2], sp[3]);
    }
    cp_async_wait<0>();
    __syncthreads();
    if (threadIdx.x < kTileRows * 8) {
        const int rr = threadIdx.x >> 3, c = threadIdx.x & 7;
        if (c < ncols_s) {
            float acc = 0.f;
            for (int st = 0; st < spu; ++st) acc = __fadd_rn(acc, stash[(st * kTileRows + rr) * 8 + c]);
            const int rowid = col_row[c];
            const int64_t t = rowid / p.top_k;
            const int k = rowid - int(t) * p.top_k;
            const int widx = p.w_index ? p.w_index[rowid] : k;
            const float wv = load_as_float(p.weights, p.w_dtype, t * p.w_tok_stride + int64_t(widx) * p.w_slot_stride);
            float cv = __fmul_rn(round_act<ACT>(acc), wv);
            if (p.w_round) cv = round_act<ACT>(cv);
            p.ybuf_g[int64_t(rowid) * p.hidden + tile * kTileRows + rr] = cv;
        }
    }
}

// ── host side ─────────────────────────────────────────────────────────────────────────────

size_t gu_smem() { return size_t(kGuWarps) * kGuDepth * 4 * 32 * sizeof(uint4); }
size_t dn_smem() { return size_t(kWarps) * kDnDepth * 2 * 32 * sizeof(uint4); }

template <typename Kernel, typename Params>
cudaError_t launch_pdl(Kernel kernel, int grid, int warps, size_t smem, cudaStream_t s, const Params& prm) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(warps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, prm);
}

// Whether the call takes the pass-per-CTA kernels: the host set a grid bound for them.
bool use_pass_kernels(const GateUpParams& gu) { return gu.max_passes > 0; }

template <int ACT, int SC, bool ZERO, int NB>
int run_decode(const GateUpParams& gu, const DownParams& dn, int sm_count, cudaStream_t s,
               cudaEvent_t const* ev, bool timed) {
    // Resident CTAs per SM of the persistent grids, from the occupancy calculator (the warp ->
    // unit assignment is static, so each whole grid must be resident at once).  The shared-memory
    // opt-in and the occupancy figures belong to the device: set up once per device.
    static int gu_per_sm[kMaxDevices], dn_per_sm[kMaxDevices];
    const int st = once_per_device(
        reinterpret_cast<const void*>(down_kernel<ACT, SC, ZERO, NB>),
        [](int dev, void*) -> int {
            cudaFuncSetAttribute(gate_up_kernel<ACT, SC, ZERO, NB, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(gu_smem()));
            cudaFuncSetAttribute(gate_up_kernel<ACT, SC, ZERO, NB, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(gu_smem()));
            cudaFuncSetAttribute(down_kernel<ACT, SC, ZERO, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(dn_smem()));
            int nblk = 0, ndn = 0;
            cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &nblk, gate_up_kernel<ACT, SC, ZERO, NB, false>, kGuWarps * 32, gu_smem());
            if (oe == cudaSuccess)
                oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ndn, down_kernel<ACT, SC, ZERO, NB>,
                                                                   kWarps * 32, dn_smem());
            if (oe != cudaSuccess || nblk < 1 || ndn < 1)
                return fail(VY_ERR_CUDA, "decode occupancy: %s", cudaGetErrorString(oe));
            gu_per_sm[dev] = nblk;
            dn_per_sm[dev] = ndn;
            return VY_OK;
        },
        nullptr);
    if (st != VY_OK) return st;
    const int dev = current_device();
    const int gu_blocks_per_sm = gu_per_sm[dev], dn_blocks_per_sm = dn_per_sm[dev];
    if constexpr (NB == 1) {
        if (gu.k_splits <= 1 && use_pass_kernels(gu)) {
            const int st2 = once_per_device(
                reinterpret_cast<const void*>(pass_gate_up_kernel<ACT, SC, ZERO>),
                [](int, void*) -> int {
                    const cudaError_t e1 = cudaFuncSetAttribute(pass_gate_up_kernel<ACT, SC, ZERO>,
                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pass_gu_smem(kRowMaxStages * kStageK)));
                    const cudaError_t e2 = cudaFuncSetAttribute(pass_down_kernel<ACT, SC, ZERO>,
                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pass_dn_smem(4 * kRowMaxStages * kStageK)));
                    return e1 == cudaSuccess && e2 == cudaSuccess ? VY_OK : fail(VY_ERR_CUDA, "pass kernels shared memory");
                },
                nullptr);
            if (st2 != VY_OK) return st2;
            cudaError_t e = launch_chained(pass_gate_up_kernel<ACT, SC, ZERO>, dim3(gu.inter / kTileRows, gu.max_passes),
                                           dim3(kPassGuWarps * 32), pass_gu_smem(gu.hidden), s, gu);
            if (e != cudaSuccess) return fail(VY_ERR_CUDA, "gate/up launch: %s", cudaGetErrorString(e));
            if (timed) cudaEventRecord(ev[2], s);
            e = launch_chained(pass_down_kernel<ACT, SC, ZERO>, dim3(dn.hidden / kTileRows, gu.max_passes),
                               dim3(kPassDnWarps * 32), pass_dn_smem(dn.inter), s, dn);
            if (e != cudaSuccess) return fail(VY_ERR_CUDA, "down launch: %s", cudaGetErrorString(e));
            return check_launch("vy_moe_decode");
        }
    }
    cudaError_t e = gu.k_splits > 1
        ? launch_pdl(gate_up_kernel<ACT, SC, ZERO, NB, true>, gu_blocks_per_sm * sm_count, kGuWarps, gu_smem(), s, gu)
        : launch_pdl(gate_up_kernel<ACT, SC, ZERO, NB, false>, gu_blocks_per_sm * sm_count, kGuWarps, gu_smem(), s, gu);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "gate/up launch: %s", cudaGetErrorString(e));
    if (timed) cudaEventRecord(ev[2], s);
    e = launch_pdl(down_kernel<ACT, SC, ZERO, NB>, dn_blocks_per_sm * sm_count, kWarps, dn_smem(), s, dn);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "down launch: %s", cudaGetErrorString(e));
    return check_launch("vy_moe_decode");
}

template <int ACT, int SC, bool ZERO>
int dispatch_nb(int nb, const GateUpParams& gu, const DownParams& dn, int sm_count,
                cudaStream_t s, cudaEvent_t const* ev, bool timed) {
    if (nb == 1) return run_decode<ACT, SC, ZERO, 1>(gu, dn, sm_count, s, ev, timed);
    if (nb == 2) return run_decode<ACT, SC, ZERO, 2>(gu, dn, sm_count, s, ev, timed);
    return run_decode<ACT, SC, ZERO, 4>(gu, dn, sm_count, s, ev, timed);
}

template <int ACT, int SC>
int dispatch_zero(bool zero, int nb, const GateUpParams& gu, const DownParams& dn, int sm_count,
                  cudaStream_t s, cudaEvent_t const* ev, bool timed) {
    return zero ? dispatch_nb<ACT, SC, true>(nb, gu, dn, sm_count, s, ev, timed)
                : dispatch_nb<ACT, SC, false>(nb, gu, dn, sm_count, s, ev, timed);
}

template <int ACT>
int dispatch_sc(int sc, bool zero, int nb, const GateUpParams& gu, const DownParams& dn, int sm_count,
                cudaStream_t s, cudaEvent_t const* ev, bool timed) {
    switch (sc) {
        case VY_BF16: return dispatch_zero<ACT, VY_BF16>(zero, nb, gu, dn, sm_count, s, ev, timed);
        case VY_F16: return dispatch_zero<ACT, VY_F16>(zero, nb, gu, dn, sm_count, s, ev, timed);
        default: return dispatch_zero<ACT, VY_F32>(zero, nb, gu, dn, sm_count, s, ev, timed);
    }
}

size_t row_gu_smem(int hidden) { return size_t(kRowGuWarps) * kRowDepth * 4 * 32 * sizeof(uint4) + size_t(hidden) * 2; }
size_t row_dn_smem() { return size_t(kRowDnWarps) * kRowDepth * 2 * 32 * sizeof(uint4); }

template <int ACT, int SC, bool ZERO>
int run_rows_typed(const RowParams& p, cudaStream_t s, cudaEvent_t const* ev, bool timed) {
    const int st = once_per_device(
        reinterpret_cast<const void*>(row_gate_up_kernel<ACT, SC, ZERO>),
        [](int, void*) -> int {
            const cudaError_t e = cudaFuncSetAttribute(row_gate_up_kernel<ACT, SC, ZERO>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(row_gu_smem(kRowMaxStages * kStageK)));
            return e == cudaSuccess ? VY_OK : fail(VY_ERR_CUDA, "few-row gate/up shared memory: %s",
                                                   cudaGetErrorString(e));
        },
        nullptr);
    if (st != VY_OK) return st;
    cudaError_t e = launch_chained(row_gate_up_kernel<ACT, SC, ZERO>, dim3(p.inter / kTileRows, p.n_rows),
                                   dim3(kRowGuWarps * 32), row_gu_smem(p.hidden), s, p);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "few-row gate/up launch: %s", cudaGetErrorString(e));
    if (timed) cudaEventRecord(ev[2], s);
    e = launch_chained(row_down_kernel<ACT, SC, ZERO>, dim3(p.hidden / kTileRows, p.n_rows), dim3(kRowDnWarps * 32),
                       row_dn_smem(), s, p);
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "few-row down launch: %s", cudaGetErrorString(e));
    return VY_OK;
}

template <int ACT>
int run_rows_act(int sc, bool zero, const RowParams& p, cudaStream_t s, cudaEvent_t const* ev, bool timed) {
    switch (sc) {
        case VY_BF16: return zero ? run_rows_typed<ACT, VY_BF16, true>(p, s, ev, timed)
                                  : run_rows_typed<ACT, VY_BF16, false>(p, s, ev, timed);
        case VY_F16: return zero ? run_rows_typed<ACT, VY_F16, true>(p, s, ev, timed)
                                 : run_rows_typed<ACT, VY_F16, false>(p, s, ev, timed);
        default: return zero ? run_rows_typed<ACT, VY_F32, true>(p, s, ev, timed)
                             : run_rows_typed<ACT, VY_F32, false>(p, s, ev, timed);
    }
}

// Whether a decode call takes the few-row kernels.
bool rows_path(const vy_moe_call* c) {
    return c->n_tokens * c->top_k <= kRowMaxRows && !c->shared_last &&
           c->geom->hidden / kStageK <= kRowMaxStages && c->geom->inter / kStageK <= kRowMaxStages;
}

struct DecodeLayout {
    int32_t *order, *live_expert, *live_start, *unit_start, *slot_order, *counters;
    PassEntry* passes;
    uint16_t *x_perm, *h_perm;
    float* ybuf_g;   // the down projection's contributions (absent when the caller takes them)
    int k_splits;    // gate/up split K (1: none)
    int64_t max_units;
    float* partial;  // k_splits > 1: per-stage partial dots of every gate/up unit
    int32_t* tickets;
    int32_t* row_tickets;   // few-row path: [n_tokens][hidden / 16] rows finished, for the combine
    size_t bytes;
};

// Column blocks (8 tokens each) one pass of a unit holds.  One block wins nearly everywhere it
// was measured (B200: cfg1 up to 16 rows per expert, cfg3, Mixtral from 6 rows per expert): the
// lighter kernels keep more warps resident than a second pass over L2-warm weights costs.  Two
// blocks win (3-7 %) only for few experts with at most 4 rows each; four never did.
int nb_for(const vy_moe_call* c) {
    const int64_t rows = c->n_tokens * c->top_k;
    return (c->n_experts <= 16 && rows <= 4 * int64_t(c->n_experts)) ? 2 : 1;
}
int call_nb(const vy_moe_call* c) { return c->col_blocks ? c->col_blocks : nb_for(c); }

// Gate/up warps of one resident wave on a 148-SM B200 (2 CTAs of kGuWarps): the split rule's
// budget.  A fixed figure, so workspace sizing and launch agree on any device.
constexpr int64_t kSplitWarps = 2 * 148 * kGuWarps;

// Gate/up split K: when even the largest possible number of (pass, tile) units leaves three
// quarters of the warps idle (batches of a token or two), each unit's K range is shared by 4 or 8
// warps, as many as keep the units within one wave and every split at least two stages long.
// (Measured on B200, cfg1: T = 1 38.1 -> 32.3 us with 4; a 2-way split at T = 2 cost more in
// partial stores and the ordered join than it gained.)
int k_splits_for(const vy_moe_call* c, int64_t max_units) {
    if (c->k_splits) return c->k_splits;
    const int spu = c->geom->hidden / kStageK;
    int s = 1;
    while (s < 8 && max_units * 2 * s <= kSplitWarps && spu % (2 * s) == 0 && spu / (2 * s) >= 2) s *= 2;
    return s >= 4 ? s : 1;
}

DecodeLayout decode_layout(const vy_moe_call* c, void* base) {
    const int64_t n = c->n_tokens * c->top_k;
    const int E = c->n_experts;
    const int64_t H = c->geom->hidden, I = c->geom->inter;
    Carve cv{static_cast<char*>(base), 0};
    DecodeLayout L{};
    L.order = cv.take<int32_t>(n);
    L.live_expert = cv.take<int32_t>(E);
    L.live_start = cv.take<int32_t>(E + 1);
    L.unit_start = cv.take<int32_t>(E + 1);
    L.slot_order = cv.take<int32_t>(n);
    L.counters = cv.take<int32_t>(4);
    const int64_t tpu = call_nb(c) * 8, max_live = n < E ? n : E;
    const int64_t max_passes = n / tpu + max_live + 1;
    L.passes = cv.take<PassEntry>(max_passes);
    L.x_perm = cv.take<uint16_t>(c->n_tokens * H);
    L.h_perm = cv.take<uint16_t>(n * I);
    L.ybuf_g = c->contrib == nullptr ? cv.take<float>(n * H) : nullptr;
    L.max_units = max_passes * (I / kTileRows);
    L.partial = nullptr;
    L.tickets = nullptr;
    L.row_tickets = nullptr;
    if (rows_path(c)) {
        // the few-row kernels: no split-K partials; one combine ticket per (token, 16-column tile)
        L.k_splits = 1;
        L.row_tickets = cv.take<int32_t>(c->n_tokens * (H / kTileRows));
        L.bytes = cv.used;
        return L;
    }
    L.k_splits = k_splits_for(c, L.max_units);
    if (L.k_splits > 1) {
        L.partial = cv.take<float>(L.max_units * (H / kStageK) * 32 * 8 * call_nb(c));
        L.tickets = cv.take<int32_t>(L.max_units);
    }
    L.bytes = cv.used;
    return L;
}

}  // namespace

// Shared validation of a vy_moe_call (decode and prefill).
int validate_call(const vy_moe_call* c) {
    if (!c || !c->geom) return fail(VY_ERR_INVALID, "null call or geometry");
    const vy_expert_geom& g = *c->geom;
    if (g.bits != 4) return fail(VY_ERR_UNSUPPORTED, "bits %d: the expert kernels take int4", g.bits);
    if (g.group_size < 32 || (g.group_size & (g.group_size - 1)))
        return fail(VY_ERR_UNSUPPORTED, "group size %d (a power of two >= 32)", g.group_size);
    if (g.hidden <= 0 || g.inter <= 0 || g.hidden % 128 || g.inter % 128)
        return fail(VY_ERR_UNSUPPORTED, "hidden %d / intermediate %d: both must be multiples of 128",
                    g.hidden, g.inter);
    if (g.hidden % g.group_size || g.inter % g.group_size)
        return fail(VY_ERR_UNSUPPORTED, "group size %d does not divide hidden %d / intermediate %d",
                    g.group_size, g.hidden, g.inter);
    if (g.scale_dtype != VY_BF16 && g.scale_dtype != VY_F16 && g.scale_dtype != VY_F32)
        return fail(VY_ERR_UNSUPPORTED, "scale dtype %d", g.scale_dtype);
    for (int r = 0; r < 3; ++r)
        if (g.word_off[r] % 4 || g.word_off[r] < 0)
            return fail(VY_ERR_ALIGNMENT, "role %d starts at word %lld (not 16-byte aligned)", r,
                        (long long)g.word_off[r]);
    if (c->act_dtype != VY_BF16 && c->act_dtype != VY_F16)
        return fail(VY_ERR_UNSUPPORTED, "activation dtype %d (bf16 / fp16)", c->act_dtype);
    if (c->w_dtype != VY_BF16 && c->w_dtype != VY_F16 && c->w_dtype != VY_F32)
        return fail(VY_ERR_UNSUPPORTED, "routing-weight dtype %d", c->w_dtype);
    if (c->ids_dtype != VY_I32 && c->ids_dtype != VY_I64)
        return fail(VY_ERR_UNSUPPORTED, "expert-id dtype %d", c->ids_dtype);
    if (c->col_blocks != 0 && c->col_blocks != 1 && c->col_blocks != 2 && c->col_blocks != 4)
        return fail(VY_ERR_UNSUPPORTED, "col_blocks %d (0, 1, 2 or 4)", c->col_blocks);
    if (c->ids_row_stride != 0 && c->ids_row_stride < c->top_k)
        return fail(VY_ERR_INVALID, "ids_row_stride %lld < top_k %d", (long long)c->ids_row_stride, c->top_k);
    int st = plan_validate(c->n_tokens, c->top_k, c->n_experts);
    if (st != VY_OK) return st;
    const int64_t n = c->n_tokens * c->top_k;
    if (c->n_tokens * int64_t(g.hidden) >= (int64_t(1) << 31) || n * int64_t(g.inter) >= (int64_t(1) << 31) ||
        n * int64_t(g.hidden) >= (int64_t(1) << 31))
        return fail(VY_ERR_UNSUPPORTED, "call too large for 32-bit element offsets");
    if (c->k_splits != 0 && c->k_splits != 1 && c->k_splits != 2 && c->k_splits != 4 && c->k_splits != 8)
        return fail(VY_ERR_INVALID, "k_splits %d (0, 1, 2, 4 or 8)", c->k_splits);
    if (c->k_splits > 1 && (g.hidden / 128) % c->k_splits)
        return fail(VY_ERR_INVALID, "k_splits %d does not divide the %d 128-element stages of hidden %d",
                    c->k_splits, g.hidden / 128, g.hidden);
    if (c->shared_last != 0 && c->shared_last != 1)
        return fail(VY_ERR_INVALID, "shared_last %d (0 or 1)", c->shared_last);
    if (c->shared_last && (c->contrib || c->top_k < 2))
        return fail(VY_ERR_INVALID, "shared_last needs the layer's own combine (contrib NULL) and top_k >= 2");
    if (c->n_tokens > 0) {
        if (!c->x || !c->expert_table || !c->expert_ids || !c->weights)
            return fail(VY_ERR_INVALID, "null input pointer");
        if (!c->out && !c->contrib && !c->shared_last) return fail(VY_ERR_INVALID, "neither out nor contrib given");
        if (c->x_row_stride < g.hidden) return fail(VY_ERR_INVALID, "x row stride %lld", (long long)c->x_row_stride);
        if (c->out && !c->contrib && c->out_row_stride < g.hidden)
            return fail(VY_ERR_INVALID, "out row stride %lld", (long long)c->out_row_stride);
        if (c->shared_last && (!c->result || c->result_row_stride < g.hidden))
            return fail(VY_ERR_INVALID, "shared_last: result %p, row stride %lld", c->result,
                        (long long)c->result_row_stride);
    }
    return VY_OK;
}

}  // namespace vy

using namespace vy;

extern "C" int vy_moe_error_flags(const vy_moe_call* c, int32_t path, int32_t* out, void* stream) {
    int st;
    if (!device_info(&st)) return st;
    if (!c || !c->geom || !out) return fail(VY_ERR_INVALID, "null call or output");
    if (!c->workspace && path != 0) return fail(VY_ERR_INVALID, "null workspace");
    const int32_t* flags;
    if (path == 1) {
        flags = prefill_flags(c);
    } else {
        // no workspace: the call ran through vy_moe_decode_static, whose scratch is the library's array
        void* ws = c->workspace;
        int st2;
        if (!ws && (st2 = decode_static_scratch(&ws)) != VY_OK) return st2;
        char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
        flags = decode_layout(c, base).counters + 2;
    }
    const cudaError_t e = cudaMemcpyAsync(out, flags, sizeof(int32_t), cudaMemcpyDefault, as_stream(stream));
    if (e != cudaSuccess) return fail(VY_ERR_CUDA, "error-flag copy: %s", cudaGetErrorString(e));
    return VY_OK;
}

extern "C" size_t vy_moe_workspace_size(const vy_moe_call* call, int32_t path) {
    if (!call || !call->geom) return 0;
    if (path == 1) return prefill_workspace_bytes(call);
    return decode_layout(call, nullptr).bytes + 256;
}

extern "C" int vy_moe_decode(const vy_moe_call* call, void* stream) {
    int st;
    const DeviceInfo* dev = device_info(&st);
    if (!dev) return st;
    if ((st = validate_call(call)) != VY_OK) return st;
    if (call->n_tokens == 0) return ok();
    const vy_moe_call* c = call;
    DecodeLayout L = decode_layout(c, nullptr);
    vy_moe_call unsplit;
    if (c->workspace && c->workspace_bytes < L.bytes + 256 && c->k_splits == 0 && L.k_splits > 1) {
        // a workspace sized for a larger batch may miss the split-K partials of a few-token call:
        // such a call runs unsplit (same result) instead of failing
        unsplit = *c;
        unsplit.k_splits = 1;
        c = &unsplit;
        L = decode_layout(c, nullptr);
    }
    if (!c->workspace || c->workspace_bytes < L.bytes + 256)
        return fail(VY_ERR_WORKSPACE, "workspace %zu bytes, %zu needed", c->workspace_bytes, L.bytes + 256);
    char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(c->workspace) + 255) & ~uintptr_t(255));
    L = decode_layout(c, base);
    const vy_expert_geom& g = *c->geom;
    cudaStream_t s = as_stream(stream);
    const int nb = call_nb(c);
    cudaEvent_t const* ev = reinterpret_cast<cudaEvent_t const*>(c->stage_events);
    const bool timed = ev != nullptr && c->n_stage_events >= 4;
    if (timed && cudaEventRecord(ev[0], s) != cudaSuccess)
        return fail(VY_ERR_INVALID, "stage_events[0] is not a usable cudaEvent_t");

    if (rows_path(c)) {
        RowParams rp{};
        rp.ids = c->expert_ids;
        rp.ids64 = c->ids_dtype == VY_I64;
        rp.ids_stride = c->ids_row_stride ? c->ids_row_stride : c->top_k;
        rp.id_base = c->expert_base;
        rp.n_experts = c->n_experts;
        rp.top_k = c->top_k;
        rp.n_rows = static_cast<int>(c->n_tokens * c->top_k);
        rp.table = c->expert_table;
        rp.hidden = g.hidden;
        rp.inter = g.inter;
        int gs_shift = 0;
        while ((1 << gs_shift) < g.group_size) ++gs_shift;
        rp.gs_shift = gs_shift;
        for (int m = 0; m < 3; ++m) {
            rp.w_off[m] = g.word_off[m];
            rp.s_off[m] = g.scale_off[m];
            rp.z_off[m] = g.zero_off[m];
        }
        rp.x = c->x;
        rp.x_stride = c->x_row_stride;
        rp.x_vec = aligned16(c->x) && (c->x_row_stride % 8 == 0);
        rp.h_perm = L.h_perm;
        rp.h_out = static_cast<uint16_t*>(c->h_out);
        rp.weights = c->weights;
        rp.w_dtype = c->w_dtype;
        rp.w_round = c->w_dtype == c->act_dtype;
        rp.w_tok_stride = c->w_tok_stride;
        rp.w_slot_stride = c->w_slot_stride;
        rp.w_index = c->w_index;
        rp.contrib = c->contrib ? c->contrib : L.ybuf_g;
        rp.flags = L.counters + 2;
        rp.out = c->contrib ? nullptr : c->out;      // the combine runs inside the down kernel
        rp.out_stride = c->out_row_stride;
        rp.tickets = L.row_tickets;
        if (timed) cudaEventRecord(ev[1], s);
        st = c->act_dtype == VY_BF16 ? run_rows_act<VY_BF16>(g.scale_dtype, g.has_zero != 0, rp, s, ev, timed)
                                     : run_rows_act<VY_F16>(g.scale_dtype, g.has_zero != 0, rp, s, ev, timed);
        if (st != VY_OK) return st;
        if (timed) cudaEventRecord(ev[3], s);
        return check_launch("vy_moe_decode");
    }

    PlanArgs pa{};
    pa.ids = c->expert_ids;
    pa.ids64 = c->ids_dtype == VY_I64;
    pa.ids_stride = c->ids_row_stride ? c->ids_row_stride : c->top_k;
    pa.id_base = c->expert_base;
    pa.n_tokens = c->n_tokens;
    pa.top_k = c->top_k;
    pa.n_experts = c->n_experts;
    pa.order = L.order;
    pa.live_expert = L.live_expert;
    pa.live_start = L.live_start;
    pa.unit_start = L.unit_start;
    pa.slot_order = L.slot_order;
    pa.counters = L.counters;
    pa.tok_per_unit = nb * 8;
    pa.x = c->x;
    pa.x_stride = c->x_row_stride;
    pa.x_vec = aligned16(c->x) && (c->x_row_stride % 8 == 0);
    pa.hidden = g.hidden;
    pa.x_perm = L.x_perm;
    pa.expert_table = c->expert_table;
    pa.passes = L.passes;
    if (L.k_splits > 1) {              // the split-K tickets start from zero every call
        pa.zero_ints = L.tickets;
        pa.zero_count = static_cast<int>(L.max_units);
    }
    if ((st = launch_plan(pa, dev->sm_count, s)) != VY_OK) return st;
    if (timed) cudaEventRecord(ev[1], s);

    int gs_shift = 0;
    while ((1 << gs_shift) < g.group_size) ++gs_shift;

    GateUpParams gu{};
    gu.hidden = g.hidden;
    gu.inter = g.inter;
    gu.gs_shift = gs_shift;
    gu.top_k = c->top_k;
    gu.w_off[0] = g.word_off[0];
    gu.w_off[1] = g.word_off[1];
    gu.s_off[0] = g.scale_off[0];
    gu.s_off[1] = g.scale_off[1];
    gu.z_off[0] = g.zero_off[0];
    gu.z_off[1] = g.zero_off[1];
    gu.passes = L.passes;
    gu.unit_start = L.unit_start;
    gu.counters = L.counters;
    gu.x_perm = L.x_perm;
    gu.h_perm = L.h_perm;
    gu.h_out = static_cast<uint16_t*>(c->h_out);
    gu.k_splits = L.k_splits;
    // Pass-per-CTA kernels for a few passes of many experts (cfg1 at 3 / 8 tokens: 44.0 -> 39.3
    // and 72.2 -> 64.7 us on B200); the warp-unit kernels from 16 tokens on (cfg1 T = 16: 99.6
    // against 105.5, T = 32: 123.5 against 125.9) and for few large experts, not measured there.
    const bool pass_ctas = nb == 1 && L.k_splits <= 1 && c->n_tokens * c->top_k <= kPassMaxRows &&
                           c->n_experts >= 64 && g.hidden / kStageK <= kRowMaxStages &&
                           g.inter / kStageK <= 4 * kRowMaxStages;
    gu.max_passes = pass_ctas ? static_cast<int>(L.max_units / (g.inter / kTileRows)) : 0;
    gu.partial = L.partial;
    gu.tickets = L.tickets;

    DownParams dn{};
    dn.hidden = g.hidden;
    dn.inter = g.inter;
    dn.gs_shift = gs_shift;
    dn.top_k = c->top_k;
    dn.w_off = g.word_off[2];
    dn.s_off = g.scale_off[2];
    dn.z_off = g.zero_off[2];
    dn.passes = L.passes;
    dn.unit_start = L.unit_start;
    dn.counters = L.counters;
    dn.h_perm = L.h_perm;
    dn.weights = c->weights;
    dn.w_dtype = c->w_dtype;
    dn.w_round = c->w_dtype == c->act_dtype;
    dn.w_tok_stride = c->w_tok_stride;
    dn.w_slot_stride = c->w_slot_stride;
    dn.w_index = c->w_index;
    dn.ybuf_g = c->contrib ? c->contrib : L.ybuf_g;

    const int sm_count = dev->sm_count;
    const bool zero = g.has_zero != 0;
    st = c->act_dtype == VY_BF16 ? dispatch_sc<VY_BF16>(g.scale_dtype, zero, nb, gu, dn, sm_count, s, ev, timed)
                                 : dispatch_sc<VY_F16>(g.scale_dtype, zero, nb, gu, dn, sm_count, s, ev, timed);
    if (st != VY_OK) return st;
    // each token's row: its slots' contributions in ascending expert id, then slot
    if (!c->contrib && (st = launch_layer_combine(c, L.ybuf_g, L.slot_order, s)) != VY_OK) return st;
    if (timed) cudaEventRecord(ev[3], s);
    return check_launch("vy_moe_decode");
}
