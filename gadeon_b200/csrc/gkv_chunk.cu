// gkv_chunk.cu -- causal paged attention for prefill chunks on the 5th-gen
// tensor cores (tcgen05 + tensor memory).
//
// Replaces the prefill-chunk attention of the reference: the per-page /
// carry-chained ANE flash tiles merged on the host
// (pagedFlashBatched / pagedFlashCarry / pagedFlashCarrySingle,
// LLM/src/CoreML/PagedAttention.swift:376-495, band mask :512-529) and Metal
// attn_batch_mm (LLM/metal/Kernels.metal:1935-2012).  Row s of a chunk that
// starts at p0 sees keys [0, p0 + s]; the result equals appending the rows
// one by one and running hostFlashDecode after each (Engine.swift:1220-1224).
//
// One CTA owns one (sequence, kv head, block of qtok = 128/G query tokens):
// its M = 128 rows are the qtok tokens x G query heads of the kv head, so
// every K/V tile it stages feeds all G heads.  Keys are walked in tiles of
// 128 (two 64-key halves).  Warp roles:
//   warps 0-3  softmax: thread r owns row r.  It stages its Q row in tensor
//              memory (the A operand of Q K^T), reads its S row (128 keys)
//              from tensor memory, applies the causal mask and the online
//              softmax (exp2 domain), writes P to shared memory for the P.V
//              MMA as two fp16 parts, P_hi = fp16(p) and P_lo = fp16(p -
//              P_hi), so P.V = P_lo.V + P_hi.V keeps ~22 significant bits of
//              every weight (PLO); with GKV_ATTEND_P_F16 (PLO = false), as P
//              rounded once to fp16 and one P.V -- the arithmetic of the
//              reference's Metal attn_batch_mm, whose P is a half tile
//              multiplied by half V into fp32 (Kernels.metal:1891-1912).  The running max is raised only when it grows by
//              more than 2^8; only then is that row of O rescaled in tensor
//              memory.
//   warps 4, 5 TMA loads of K tiles (warp 4) and V tiles (warp 5), one lane
//              per page group, into ONE ring of 128-key stages that both share.
//              The ring is filled in the order the tensor core consumes it --
//              K0, K1, V0, K2, V1, K3, V2, ... -- so every load is issued two
//              MMAs ahead of its use (with separate K and V rings, V got one).
//   warp 6     owns tensor memory; one thread issues S = Q K^T
//              (tcgen05.mma M=128, N=128) and O += P V (N = dh, V read
//              MN-major, eight K=16 steps) into the fp32 O accumulator that
//              stays in tensor memory for the whole loop.
// Measured on B200: an N=64 tcgen05.mma costs as long as an N=128 one, so Q K^T
// runs with N=128.  S is single-buffered (softmax releases it as soon as it
// has read its row), so Q K^T of tile j+1 overlaps the softmax of tile j.
// Completion flows through mbarriers: tcgen05.commit for tensor-core work,
// TMA transaction counts for loads.  Every wait is bounded; a timeout raises
// the device status word.
//
// CTA pairs (PAIR = true, dh 128/256, two or more query blocks): a cluster of
// two CTAs on neighbouring SMs runs one M = 256 tile with tcgen05.mma
// cta_group::2 -- each CTA holds its own 128 rows (Q, S, O in its tensor
// memory, P in its shared memory) and loads HALF of every K tile (64 of the
// 128 keys) and HALF of every V tile (dh/2 of the head-dim columns); the
// tensor cores of the pair exchange the halves.  Each SM then streams half
// the K/V bytes per FLOP.  The even CTA issues every MMA; its commits arrive
// on both CTAs' barriers, the odd CTA's loads complete on the even CTA's
// barriers, and the odd CTA's softmax warps arrive remotely on them.
#include <atomic>
#include <cuda_fp16.h>

#include "gkv_kernels.cuh"
#include "gkv_ptx.cuh"

namespace gkv {
namespace {

using namespace ptx;

constexpr int kSoftmaxWarps = 4;
constexpr int kChunkThreads = (kSoftmaxWarps + 3) * 32;
constexpr int kKWarp = 4, kVWarp = 5, kMmaWarp = 6;
constexpr int kChunkRows = 128;   // tensor-memory lanes = rows per CTA
constexpr int kHalf = 64;         // keys per P atom; most rows in one TMA box
constexpr int kTile = 2 * kHalf;  // keys per tile (tcgen05 N of Q K^T)
constexpr uint32_t kTmemMaxCols = 512;  // tensor memory columns per SM
constexpr int kSmemLimit = 227 * 1024;

template <int DH, bool PAIR, bool PLO>
struct ChunkCfg {
    static constexpr int NCB = DH / 64;
    static_assert(!PAIR || NCB >= 2, "a CTA pair splits V by 64-column blocks");
    // A stage holds this CTA's part of one 128-key tile of K or V, 64-column
    // blocks of 128-byte rows (128B swizzle, 8-row groups 1024 bytes apart).
    // K (read K-major, the B operand of Q K^T): NCB blocks of K_ROWS keys --
    // all 128 keys, or this CTA's 64 in a pair.  V (read MN-major, the B
    // operand of P V, block stride as LBO): V_NCB blocks of 128 keys -- all
    // head-dim blocks, or this CTA's half in a pair.  Both fill a stage.
    static constexpr int K_ROWS = PAIR ? kHalf : kTile;
    static constexpr int CB_K = K_ROWS * 128;
    static constexpr int V_NCB = PAIR ? NCB / 2 : NCB;
    static constexpr int CB_V = kTile * 128;
    static constexpr int STAGE_BYTES = NCB * CB_K;
    static_assert(STAGE_BYTES == V_NCB * CB_V, "K and V parts fill the same stage");
    // P as P_hi and P_lo (fp16 each, two 64-key atoms each): P.V runs as
    // P_hi.V + P_lo.V so the weights keep ~22 significant bits (PLO); or P
    // rounded once to fp16 and one P.V (GKV_ATTEND_P_F16)
    static constexpr int P_ONE = kChunkRows * kTile * 2;
    static constexpr int P_BYTES = PLO ? 2 * P_ONE : P_ONE;
    static constexpr int NS_FIT = (kSmemLimit - 2048 - P_BYTES) / STAGE_BYTES;
    static constexpr int NS = NS_FIT < 8 ? NS_FIT : 8;      // ring depth
    static_assert(NS >= 3, "the ring needs three stages");
    static constexpr int OFF_STAGE = 0;
    static constexpr int OFF_P = OFF_STAGE + NS * STAGE_BYTES;  // P_hi
    static constexpr int OFF_PL = OFF_P + P_ONE;                  // P_lo (PLO only)
    static constexpr int OFF_BAR = OFF_P + P_BYTES;
    static constexpr int NBARS = 2 * NS + 5;
    static constexpr int SMEM = OFF_BAR + NBARS * 8 + 16;
    // Tensor memory: S (128 fp32 columns), O (dh fp32 columns), Q (dh fp16 =
    // dh/2 columns, the A operand of Q K^T).
    static constexpr uint32_t O_COL = kTile;
    static constexpr uint32_t Q_COL = O_COL + DH;
    static constexpr uint32_t USED_COLS = Q_COL + DH / 2;
    static constexpr uint32_t TMEM_COLS = USED_COLS <= 256 ? 256 : 512;
    static_assert(USED_COLS <= TMEM_COLS, "S, O and Q fit tensor memory");
    // Co-resident CTAs must not ask for more than the SM's 512 columns,
    // else tcgen05.alloc would wait for a neighbour to finish: pad the
    // shared-memory request so at most 512 / TMEM_COLS CTAs fit on an SM.
    static constexpr int MIN_SMEM = (228 * 1024) / (int)(kTmemMaxCols / TMEM_COLS + 1) + 1024;
    static constexpr int SMEM_ALLOC = SMEM + 1024 > MIN_SMEM ? SMEM + 1024 : MIN_SMEM;
    static_assert(SMEM_ALLOC <= kSmemLimit, "fits the per-CTA shared memory limit");
};

template <int DH, bool PAIR, bool PLO>
__global__ void __launch_bounds__(kChunkThreads, 1)
    chunk_kernel(const __grid_constant__ ChunkParams p, const __grid_constant__ CUtensorMap tmk,
                 const __grid_constant__ CUtensorMap tmv) {
    using C = ChunkCfg<DH, PAIR, PLO>;
    constexpr int M = kChunkRows, TT = kTile, H = kHalf;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *full = bars;                    // [NS] TMA -> MMA (the even CTA's count both halves)
    uint64_t *empty = bars + C::NS;           // [NS] MMA commit -> loaders
    uint64_t *s_full = bars + 2 * C::NS;      // MMA commit -> softmax
    uint64_t *s_free = bars + 2 * C::NS + 1;  // softmax warps (of both CTAs) -> MMA
    uint64_t *p_full = bars + 2 * C::NS + 2;  // softmax warps (of both CTAs) -> MMA
    uint64_t *p_free = bars + 2 * C::NS + 3;  // MMA commit (P.V done) -> softmax
    uint64_t *vtail = bars + 2 * C::NS + 4;   // pair: this CTA's part of the last V tile landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    // longest key ranges first; a pair takes two consecutive query blocks
    const int qb = PAIR ? 2 * ((p.n_qblocks + 1) / 2 - 1 - (int)(blockIdx.x >> 1)) + (int)rank
                        : p.n_qblocks - 1 - (int)blockIdx.x;
    const int kvh = blockIdx.y, b = blockIdx.z;
    const AttendEntry e = p.entries[b];
    const int G = p.G, KVH = p.kvh;
    const int p0 = e.len - p.n_q;
    // t_hi < t_lo (no valid rows) for a pair's odd block past the chunk's end
    const int t_lo = qb * p.qtok, t_hi = min(p.n_q, t_lo + p.qtok);
    const int kend = p0 + (PAIR ? min(p.n_q, (qb - (int)rank + 2) * p.qtok) : t_hi);  // keys [0, kend)
    const int nt = (kend + TT - 1) / TT;
    // position of tile j's K and V in the ring's fill sequence K0 K1 V0 K2 V1 ...
    auto kidx = [&](int j) { return j == 0 ? 0 : 2 * j - 1; };
    auto vidx = [&](int j) { return min(2 * j + 2, 2 * nt - 1); };
    auto stage = [&](int idx) { return smem + C::OFF_STAGE + (idx % C::NS) * C::STAGE_BYTES; };
    // waits on barriers that the other CTA of a pair also arrives on acquire at cluster scope
    auto wait = [&](uint64_t *bar, uint32_t parity) {
        if constexpr (PAIR)
            return mbar_wait_cluster(bar, parity, abort_flag, p.status);
        else
            return mbar_wait(bar, parity, abort_flag, p.status);
    };
    // softmax -> MMA arrivals land on the even CTA's barrier
    auto arrive_leader = [&](uint64_t *bar) {
        if (PAIR && !leader)
            mbar_arrive_cluster(mapa_shared(smem_u32(bar), 0));
        else
            mbar_arrive(bar);
    };

    if (tid == 0) {
        for (int i = 0; i < 2 * C::NS; ++i) mbar_init(&bars[i], 1);
        mbar_init(s_full, 1);
        mbar_init(s_free, (PAIR ? 2 : 1) * kSoftmaxWarps);
        mbar_init(p_full, (PAIR ? 2 : 1) * kSoftmaxWarps);
        mbar_init(p_free, 1);
        mbar_init(vtail, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, C::TMEM_COLS);
            tmem_relinquish();
        }
    }
    // K/V stages start zeroed so never-loaded slots hold finite values.
    for (int i = tid; i < (C::OFF_P - C::OFF_STAGE) / 16; i += kChunkThreads)
        reinterpret_cast<uint4 *>(smem + C::OFF_STAGE)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Q into tensor memory: softmax thread r writes row r = token t_lo + r/G,
    // head kvh*G + r%G as dh/2 packed fp16 pairs (padding rows zero).
    if (warp < kSoftmaxWarps) {
        const int t = tid / G, g = tid - t * G, tok = t_lo + t;
        const bool valid = t < p.qtok && tok < t_hi;
        const uint4 *src = reinterpret_cast<const uint4 *>(
            p.q + qo_row(p.head_major, b, valid ? tok : 0, kvh, g, p.n_q, KVH, G) * DH);
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16) + C::Q_COL;
#pragma unroll 1
        for (int c0 = 0; c0 < DH / 2; c0 += 32) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 x = valid ? src[c0 / 4 + i] : make_uint4(0u, 0u, 0u, 0u);
                v[4 * i] = __uint_as_float(x.x);
                v[4 * i + 1] = __uint_as_float(x.y);
                v[4 * i + 2] = __uint_as_float(x.z);
                v[4 * i + 3] = __uint_as_float(x.w);
            }
            tmem_st32(trow + c0, v);
        }
        tmem_wait_st();
    }
    // Both CTAs' Q rows and barriers are in place before the first MMA or
    // remote arrival.
    tc_fence_before();
    __syncwarp();
    if constexpr (PAIR)
        cluster_sync();
    else
        __syncthreads();
    tc_fence_after();

    if (warp == kKWarp || warp == kVWarp) {
        // ============================================ TMA producers
        // Lane i of the warp owns page group i of this CTA's part of a tile
        // (group = min(P, 64) keys of one page).  Every lane reads its
        // block-table entry before the stage wait, in parallel, so the table
        // latency is paid once per tile instead of once per page; then each
        // lane issues its own group's boxes (one per 64-column block).
        const bool is_k = warp == kKWarp;
        const CUtensorMap *map = is_k ? &tmk : &tmv;
        const int lP = __ffs(p.P) - 1;
        const int bh = min(p.P, H);
        const int32_t *trow = p.table + (int64_t)e.seq_id * p.table_stride;
        const int key_cnt = (PAIR && is_k) ? H : TT;            // keys of a tile this CTA loads
        const int key_off = (PAIR && is_k) ? (int)rank * H : 0;
        const int ncb = is_k ? C::NCB : C::V_NCB;               // 64-column blocks it loads
        const int cb_lo = (PAIR && !is_k) ? (int)rank * C::V_NCB : 0;
        const int cb_bytes = is_k ? C::CB_K : C::CB_V;
        auto part_bytes = [&](int t0, int r) {  // bytes CTA r loads of the tile at t0
            const int n = max(0, min(key_cnt, kend - t0 - ((PAIR && is_k) ? r * H : 0)));
            return (uint32_t)(((n + bh - 1) / bh) * bh * ncb * 128);
        };
        for (int j = 0; j < nt; ++j) {
            const int idx = is_k ? kidx(j) : vidx(j);
            const int st = idx % C::NS;
            const int t0 = j * TT;
            const int tg = t0 + key_off + lane * bh;
            const bool mine = lane < key_cnt / bh && tg < kend;
            // pair: each CTA counts its part of the last V tile on its own
            // barrier, so its softmax warps can zero the rows past the end
            const bool tail = PAIR && !is_k && j == nt - 1;
            int row0 = 0;
            if (mine) {
                int pid = __ldg(trow + (tg >> lP));
                if (pid < 0 || pid >= p.num_pages) {
                    atomicOr(p.status, DEV_ERR_BAD_PAGE);
                    pid = 0;
                }
                row0 = (pid * KVH + kvh) * p.P + (tg & (p.P - 1));
            }
            bool ok = true;
            if (lane == 0) {
                if (idx >= C::NS) ok = mbar_wait(&empty[st], ((idx / C::NS) - 1) & 1, abort_flag, p.status);
                if (ok) {
                    if (tail)
                        mbar_expect_tx(vtail, part_bytes(t0, (int)rank));
                    else if (leader)
                        mbar_expect_tx(&full[st], PAIR ? part_bytes(t0, 0) + part_bytes(t0, 1) : part_bytes(t0, 0));
                }
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            if (mine) {
                const uint32_t dst = smem_u32(stage(idx)) + (uint32_t)(lane * bh * 128);
                const uint32_t lead_bar = PAIR && !leader && !tail ? mapa_shared(smem_u32(&full[st]), 0) : 0u;
                for (int c = 0; c < ncb; ++c) {
                    const uint32_t d = dst + (uint32_t)(c * cb_bytes);
                    const int x = (cb_lo + c) * 64;
                    if (tail)
                        tma_load_2d(d, map, x, row0, vtail);
                    else if (!PAIR || leader)
                        tma_load_2d(d, map, x, row0, &full[st]);
                    else
                        tma_load_2d_pair(d, map, x, row0, lead_bar);
                }
            }
            __syncwarp();
        }
    } else if (warp == kMmaWarp) {
        // ============================================ MMA issue (lane 0 of the even CTA)
        if (lane == 0 && leader) {
            constexpr int MM = PAIR ? 2 * M : M;
            constexpr uint32_t IDESC_QK = umma_idesc_f16(MM, TT, 0);
            constexpr uint32_t IDESC_PV = umma_idesc_f16(MM, DH, 1);
            auto commit = [&](uint64_t *bar) {  // this CTA's barrier and the peer's
                if constexpr (PAIR) {
                    umma_pair_commit(smem_u32(bar));
                    umma_pair_commit(mapa_shared(smem_u32(bar), 1));
                } else {
                    umma_commit(bar);
                }
            };
            auto issue_pv = [&](int i) -> bool {
                const int vi = vidx(i);
                if (!wait(p_full, i & 1)) return false;
                // a pair's last V tile is covered by p_full: each softmax
                // group waited for its CTA's part before arriving
                if (!(PAIR && i == nt - 1) && !wait(&full[vi % C::NS], (vi / C::NS) & 1)) return false;
                tc_fence_after();
                const uint32_t sV = smem_u32(stage(vi));
                const uint32_t sP = smem_u32(smem + C::OFF_P);
                [[maybe_unused]] const uint32_t sPl = smem_u32(smem + C::OFF_PL);
#pragma unroll
                for (int kk = 0; kk < TT / 16; ++kk) {
                    // P atom kk/4 holds keys 64*(kk/4) .. +63; V is MN-major:
                    // 64-column blocks CB_V apart (LBO), 8-key groups 1024
                    // bytes apart (SBO), 16 keys = 2048 bytes per K step.
                    const uint32_t patom = (kk >> 2) * M * 128 + (kk & 3) * 32;
                    const uint64_t a = umma_desc_sw128(sP + patom, 16, 1024);
                    [[maybe_unused]] const uint64_t al = umma_desc_sw128(sPl + patom, 16, 1024);
                    const uint64_t bd = umma_desc_sw128(sV + kk * 16 * 128, C::CB_V, 1024);
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    if constexpr (PLO) {
                        if constexpr (PAIR) {
                            umma_pair_f16(tmem + C::O_COL, al, bd, IDESC_PV, acc);
                            umma_pair_f16(tmem + C::O_COL, a, bd, IDESC_PV, 1u);
                        } else {
                            umma_f16(tmem + C::O_COL, al, bd, IDESC_PV, acc);
                            umma_f16(tmem + C::O_COL, a, bd, IDESC_PV, 1u);
                        }
                    } else {
                        if constexpr (PAIR)
                            umma_pair_f16(tmem + C::O_COL, a, bd, IDESC_PV, acc);
                        else
                            umma_f16(tmem + C::O_COL, a, bd, IDESC_PV, acc);
                    }
                }
                commit(&empty[vi % C::NS]);
                commit(p_free);
                return true;
            };
            bool ok = true;
            for (int j = 0; j < nt && ok; ++j) {
                const int ki = kidx(j);
                ok = wait(&full[ki % C::NS], (ki / C::NS) & 1) && (j < 1 || wait(s_free, (j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const uint32_t sK = smem_u32(stage(ki));
#pragma unroll
                for (int ks = 0; ks < DH / 16; ++ks) {  // A = Q from tensor memory, 8 columns per K=16
                    const uint64_t bd = umma_desc_sw128(sK + (ks >> 2) * C::CB_K + (ks & 3) * 32, 16, 1024);
                    if constexpr (PAIR)
                        umma_pair_f16_ts(tmem, tmem + C::Q_COL + ks * 8, bd, IDESC_QK, ks > 0);
                    else
                        umma_f16_ts(tmem, tmem + C::Q_COL + ks * 8, bd, IDESC_QK, ks > 0);
                }
                commit(s_full);
                commit(&empty[ki % C::NS]);
                if (j >= 1) ok = issue_pv(j - 1);
            }
            if (ok) issue_pv(nt - 1);
        }
    } else {
        // ============================================ softmax warps
        const int r = tid;
        const uint32_t tmem_row = tmem + ((uint32_t)(warp * 32) << 16);
        const int tr = r / G, tok = t_lo + tr;
        const bool row_valid = tr < p.qtok && tok < t_hi;
        const int lim = row_valid ? p0 + tok : p0;  // last visible key
        const int all_visible = p0 + t_lo;           // keys <= this are visible to every row
        const float sl = p.scale_log2;
        const float sgn = sl >= 0.f ? 1.f : -1.f;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            if (!wait(s_full, j & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s[TT];  // this row's 128 raw scores
#pragma unroll
            for (int q4 = 0; q4 < TT / 32; ++q4) {
                float (&part)[32] = *reinterpret_cast<float (*)[32]>(&s[q4 * 32]);
                tmem_ld32(tmem_row + (uint32_t)(q4 * 32), part);
            }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader(s_free);

            const int t0 = j * TT;
            if (t0 + TT - 1 > all_visible) {
                // masked keys become -inf * sign(scale) so scale * s = -inf
#pragma unroll
                for (int c = 0; c < TT; ++c)
                    if (t0 + c > lim) s[c] = -INFINITY * sgn;
            }
            // extreme of the raw scores, 8 chains: the max for scale >= 0 (no
            // sign products in the usual case), the min for a negative scale
            float ex[8], ext;
#pragma unroll
            for (int u = 0; u < 8; ++u) ex[u] = s[u];
            if (sl >= 0.f) {
#pragma unroll
                for (int c = 8; c < TT; ++c) ex[c & 7] = fmaxf(ex[c & 7], s[c]);
                ext = fmaxf(fmaxf(fmaxf(ex[0], ex[1]), fmaxf(ex[2], ex[3])),
                            fmaxf(fmaxf(ex[4], ex[5]), fmaxf(ex[6], ex[7])));
            } else {
#pragma unroll
                for (int c = 8; c < TT; ++c) ex[c & 7] = fminf(ex[c & 7], s[c]);
                ext = fminf(fminf(fminf(ex[0], ex[1]), fminf(ex[2], ex[3])),
                            fminf(fminf(ex[4], ex[5]), fminf(ex[6], ex[7])));
            }
            const float mt = ext == -INFINITY * sgn ? -INFINITY : ext * sl;
            const float m_new = fmaxf(m_ref, mt);
            const bool raise = m_new > m_ref + 8.f;  // lazy: keep m_ref unless it grew by > 2^8
            float factor = 1.f;
            if (raise) {
                factor = m_ref == -INFINITY ? 0.f : fast_exp2(m_ref - m_new);
                m_ref = m_new;
            }
            const float nmu = m_ref == -INFINITY ? 0.f : -m_ref;
            if (j >= 1) {
                // P.V of tile j-1 must be done before P is rewritten or O rescaled.
                if (!wait(p_free, (j - 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, raise)) {
#pragma unroll 1
                    for (int c0 = 0; c0 < DH; c0 += 32) {
                        float o[32];
                        tmem_ld32(tmem_row + C::O_COL + c0, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= factor;
                        tmem_st32(tmem_row + C::O_COL + c0, o);
                    }
                    tmem_wait_st();
                }
            }
            uint8_t *sP = smem + C::OFF_P;
            [[maybe_unused]] uint8_t *sPl = smem + C::OFF_PL;
            // packed fp32x2 FMA / add (each lane rounded as fmaf / + would)
            float2 ps2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
            const float2 sl2 = make_float2(sl, sl), nmu2 = make_float2(nmu, nmu);
#pragma unroll
            for (int ch = 0; ch < TT / 8; ++ch) {  // 16-byte chunks of 8 keys
                uint32_t w4[4];
                [[maybe_unused]] uint32_t w4l[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float2 x = __ffma2_rn(make_float2(s[ch * 8 + 2 * u], s[ch * 8 + 2 * u + 1]), sl2, nmu2);
                    const float a0 = fast_exp2(x.x), a1 = fast_exp2(x.y);
                    ps2[u] = __fadd2_rn(ps2[u], make_float2(a0, a1));
                    if constexpr (PLO) {
                        split_half2(a0, a1, w4[u], w4l[u]);
                    } else {
                        const __half2 h = __floats2half2_rn(a0, a1);
                        w4[u] = *reinterpret_cast<const uint32_t *>(&h);
                    }
                }
                // P atom (ch / 8) holds keys 64*(ch/8) .. +63 of all rows
                const int at = (ch >> 3) * M * 128 + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
                *reinterpret_cast<uint4 *>(sP + at) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                if constexpr (PLO)
                    *reinterpret_cast<uint4 *>(sPl + at) = make_uint4(w4l[0], w4l[1], w4l[2], w4l[3]);
            }
            l = l * factor + (((ps2[0].x + ps2[0].y) + (ps2[1].x + ps2[1].y)) +
                              ((ps2[2].x + ps2[2].y) + (ps2[3].x + ps2[3].y)));
            const int nkeys = min(TT, kend - t0);
            if (j == nt - 1 && (PAIR || nkeys < TT)) {
                // last tile: once this CTA's part of V landed, zero its rows
                // past the block's end (stale data; P is 0 there, and 0 * V
                // must stay 0)
                const int vi = vidx(j);
                const bool landed = PAIR ? wait(vtail, 0) : wait(&full[vi % C::NS], (vi / C::NS) & 1);
                if (!landed) {
                    ok = false;
                    break;
                }
                uint8_t *sV = stage(vi);
                for (int i = tid; i < (TT - nkeys) * (C::V_NCB * 8); i += kSoftmaxWarps * 32) {
                    const int key = nkeys + i / (C::V_NCB * 8), c16 = i % (C::V_NCB * 8);
                    *reinterpret_cast<uint4 *>(sV + (c16 >> 3) * C::CB_V + key * 128 +
                                               (((c16 & 7) ^ (key & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_proxy_async();  // P (and V zeroing) written by threads -> tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader(p_full);
        }
        // ---- epilogue: O / l for valid rows once the last P.V is done
        if (ok && wait(p_free, (nt - 1) & 1)) {
            tc_fence_after();
            const float inv = 1.f / l;
            const int64_t at = qo_row(p.head_major, b, row_valid ? tok : 0, kvh, r - tr * G, p.n_q, KVH, G) * DH;
#pragma unroll 1
            for (int c0 = 0; c0 < DH; c0 += 32) {
                float o[32];
                tmem_ld32(tmem_row + C::O_COL + c0, o);
                tmem_wait_ld();
                if (row_valid) {
                    if (p.out_f16) {  // each value rounded to nearest even
                        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + at + c0);
#pragma unroll
                        for (int i = 0; i < 32; i += 8)
                            dst[i / 8] = make_uint4(pack_half2(o[i] * inv, o[i + 1] * inv),
                                                    pack_half2(o[i + 2] * inv, o[i + 3] * inv),
                                                    pack_half2(o[i + 4] * inv, o[i + 5] * inv),
                                                    pack_half2(o[i + 6] * inv, o[i + 7] * inv));
                    } else {
                        float *dst = static_cast<float *>(p.out) + at + c0;
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(dst + i) =
                                make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
                    }
                }
            }
        }
    }
    // No CTA of a pair frees tensor memory or leaves while the other may
    // still use it or its shared memory.
    tc_fence_before();
    __syncwarp();
    if constexpr (PAIR)
        cluster_sync();
    else
        __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        if constexpr (PAIR)
            tmem_dealloc_pair(tmem, C::TMEM_COLS);
        else
            tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int DH, bool PAIR, bool PLO>
cudaError_t launch_chunk_t(const ChunkParams &p, const CUtensorMap *tk, const CUtensorMap *tv,
                           cudaStream_t s) {
    auto kern = chunk_kernel<DH, PAIR, PLO>;
    constexpr int smem = ChunkCfg<DH, PAIR, PLO>::SMEM_ALLOC;
    static std::atomic<bool> configured[64];  // per device; setting the attribute twice is harmless
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured[dev].store(true, std::memory_order_release);
    }
    if constexpr (PAIR) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * ((p.n_qblocks + 1) / 2), p.kvh, p.n_seqs);
        cfg.blockDim = dim3(kChunkThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, p, *tk, *tv);
    } else {
        dim3 grid(p.n_qblocks, p.kvh, p.n_seqs);
        kern<<<grid, kChunkThreads, smem, s>>>(p, *tk, *tv);
        return cudaGetLastError();
    }
}

}  // namespace

bool chunk_supported(int dh, int P, int G) {
    return (dh == 64 || dh == 128 || dh == 256) && P >= 8 && G >= 1 && G <= kChunkRows;
}

// CTA pairs when the chunk has two or more query blocks and dh splits into
// two halves of whole 64-column blocks; one CTA per block otherwise.  At dh
// 256 always pairs (a lone block's partner has no rows): one CTA's 64 KB
// stages would leave room for only two beside P_hi and P_lo.
template <bool PLO>
cudaError_t launch_chunk_p(const ChunkParams &p, const CUtensorMap *tk, const CUtensorMap *tv, int dh,
                           cudaStream_t s) {
    const bool pair = p.n_qblocks >= 2;
    switch (dh) {
        case 64: return launch_chunk_t<64, false, PLO>(p, tk, tv, s);
        case 128:
            return pair ? launch_chunk_t<128, true, PLO>(p, tk, tv, s) : launch_chunk_t<128, false, PLO>(p, tk, tv, s);
        case 256: return launch_chunk_t<256, true, PLO>(p, tk, tv, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_chunk(const ChunkParams &p, const CUtensorMap *tk, const CUtensorMap *tv, int dh,
                         cudaStream_t s) {
    return p.p_f16 ? launch_chunk_p<false>(p, tk, tv, dh, s) : launch_chunk_p<true>(p, tk, tv, dh, s);
}

}  // namespace gkv
