// tsrc_fa_plan.cu -- host side of flash attention: shape rules, mask summary, chunk plan.
//
// What the reference's backend and RISC-V kernel decide before any tile op runs, restated in C++:
//   - shape checks and the pass rule GS = min(G, T_MAX), T_q = floor(T_MAX / GS)
//     (jwkim04/tesseract-npu sw/sim/tsr_ref_at.c:726-769, tsr_ref_at.h:268-277);
//   - the mask summary MSUM: per query row at most two runs of visible cells (f16 +-0), else the
//     whole call takes the GENERAL path (tsr_ref_at.c:646-692);
//   - the chunk planner, rules 1-8 of sw/sim/include/tsr_fa_plan.h: sub-ranges of visible groups,
//     the chunk size NCG = min(128, C floor(PCAP / (16 E / D)), max(4C, roundup_4C(ceil(n/2)))),
//     cuts every NCG groups, no cut inside a causal / sliding-window spread, the encoded bounds of
//     each chunk (verified against every row's runs), chunks holding a new cell last.
// The output is the list of work items (query tile x chunk) the kernels run.
#include <algorithm>
#include <cstdint>
#include <vector>

#include "../../include/tsrc.h"
#include "tsrc_internal.h"

namespace tsrc {

namespace {

constexpr uint32_t kCausal = 1u, kSlide = 2u;

struct Run {
    uint32_t lo0, hi0, lo1, hi1;
};

struct Sub {
    uint32_t ulo, uhi;
    bool general, multi;
    uint32_t flags;
    int64_t lo, hi;
};

// MSUM of the f16 mask: -inf (0xFC00) hides a cell, +-0 shows it, anything else is GENERAL.
bool summarize(const uint16_t* mask, size_t stride, uint32_t n_kv, uint32_t T, std::vector<Run>& rows) {
    bool general = false;
    rows.assign(T, Run{0, 0, 0, 0});
    for (uint32_t q = 0; q < T; ++q) {
        Run& r = rows[q];
        if (!mask) {
            r.hi0 = n_kv;
            continue;
        }
        const uint16_t* m = mask + (size_t)q * stride;
        uint32_t nrun = 0;
        for (uint32_t j = 0; j < n_kv;) {
            if (m[j] == 0xFC00u) {
                ++j;
                continue;
            }
            if (m[j] & 0x7FFFu) {
                general = true;
                ++j;
                continue;
            }
            uint32_t e = j;
            while (e < n_kv && (m[e] & 0x7FFFu) == 0) ++e;
            if (nrun == 0) {
                r.lo0 = j;
                r.hi0 = e;
            } else if (nrun == 1) {
                r.lo1 = j;
                r.hi1 = e;
            }
            ++nrun;
            j = e;
        }
        if (nrun > 2) general = true;
    }
    return general;
}

uint32_t chunk_groups(uint32_t C, uint32_t pcap, uint32_t E, uint32_t D, uint32_t n_total) {
    if (D == 0 || E % D || C == 0 || E / D == 0) return 0;
    const uint64_t by_pcap = (uint64_t)C * (pcap / (16u * (E / D)));
    if (by_pcap == 0) return 0;
    const uint64_t half = ((uint64_t)n_total + 1u) / 2u, c4 = 4u * (uint64_t)C;
    const uint64_t by_n = c4 >= half ? c4 : (half + c4 - 1u) / c4 * c4;
    return (uint32_t)std::min<uint64_t>({128u, by_pcap, by_n});
}

// The encoded bounds of chunk [a, b) of sub-range s (rule 6); false if they cannot reproduce
// every row's visible cells.
bool encode(const Sub& s, uint32_t Tq, const int64_t* L, const int64_t* H, uint32_t a, uint32_t b, FaItem& c) {
    c.u0 = a;
    c.n = b - a;
    c.flags = 0;
    c.general = 0;
    const int64_t A = 16 * (int64_t)a, n16 = 16 * (int64_t)b - A;
    if (s.general) {
        c.general = 1;
        c.c_lo = 0;
        c.c_hi = (uint32_t)n16;
        return true;
    }
    if (!s.multi) {
        c.c_lo = (uint32_t)std::max<int64_t>(s.lo - A, 0);
        c.c_hi = (uint32_t)std::min<int64_t>(s.hi - A, n16);
        return true;
    }
    int64_t clo = 0, chi = n16;
    uint32_t fl = 0;
    if (s.lo > A) {
        clo = s.lo - A;
        if (s.flags & kSlide) fl |= kSlide;
    }
    if (s.hi - ((s.flags & kCausal) ? (int64_t)Tq - 1 : 0) < A + n16) {
        chi = s.hi - A;
        if (s.flags & kCausal) fl |= kCausal;
    }
    if (clo < 0 || clo > chi || chi > n16) return false;
    for (uint32_t q = 0; q < Tq; ++q) {
        const int64_t dq = (int64_t)Tq - 1 - q;
        const int64_t lq = std::max<int64_t>(0, clo - ((fl & kSlide) ? dq : 0));
        const int64_t hq = std::min<int64_t>(chi - ((fl & kCausal) ? dq : 0), n16);
        const int64_t el = std::max<int64_t>(L[q] - A, 0), eh = std::min<int64_t>(H[q] - A, n16);
        const bool ea = hq <= lq, eb = eh <= el;
        if (ea != eb || (!ea && (lq != el || hq != eh))) return false;
    }
    c.c_lo = (uint32_t)clo;
    c.c_hi = (uint32_t)chi;
    c.flags = fl;
    return true;
}

// Chunks of the tile [q0, q0 + Tq) in execution order, appended to out. 0 or a TSRC_E_* code.
int plan_tile(const FaPlanIn& in, uint32_t E, bool general, const Run* rows, uint32_t q0, uint32_t Tq,
              std::vector<FaItem>& out, const char** why) {
    std::vector<Sub> subs;
    int64_t L[8] = {0}, H[8] = {0};
    if (general) {
        if (in.n_kv > 0) subs.push_back(Sub{0, (in.n_kv + 15u) >> 4, true, false, 0, 0, 0});
    } else {
        int64_t rl[8][2], rh[8][2];
        uint32_t nr[8];
        bool all_one = true;
        int64_t hlo = INT64_MAX, hhi = -1;
        for (uint32_t q = 0; q < Tq; ++q) {
            const Run& w = rows[q];
            uint32_t n = 0;
            if (w.hi0 > w.lo0) {
                rl[q][n] = w.lo0;
                rh[q][n] = w.hi0;
                ++n;
            }
            if (w.hi1 > w.lo1) {
                rl[q][n] = w.lo1;
                rh[q][n] = w.hi1;
                ++n;
            }
            if (n == 2 && rl[q][1] < rl[q][0]) {
                std::swap(rl[q][0], rl[q][1]);
                std::swap(rh[q][0], rh[q][1]);
            }
            nr[q] = n;
            all_one = all_one && n == 1;
            for (uint32_t k = 0; k < n; ++k) {
                hlo = std::min(hlo, rl[q][k]);
                hhi = std::max(hhi, rh[q][k]);
            }
        }
        if (Tq == 1) {
            for (uint32_t k = 0; k < nr[0]; ++k)
                subs.push_back(Sub{(uint32_t)(rl[0][k] / 16), (uint32_t)((rh[0][k] + 15) / 16), false, false, 0, rl[0][k], rh[0][k]});
        } else if (hhi >= 0) {
            bool fit = all_one;
            uint32_t fl = 0;
            int64_t lo_abs = 0, hi_abs = 0;
            if (fit) {
                for (uint32_t q = 0; q < Tq; ++q) {
                    L[q] = rl[q][0];
                    H[q] = rh[q][0];
                }
                hi_abs = H[Tq - 1];
                lo_abs = L[Tq - 1];
                bool heq = true, leq = true, hca = true, lsl = lo_abs > 0;
                for (uint32_t q = 0; q < Tq; ++q) {
                    const int64_t dq = (int64_t)Tq - 1 - q;
                    heq = heq && H[q] == hi_abs;
                    leq = leq && L[q] == lo_abs;
                    hca = hca && H[q] == hi_abs - dq;
                    lsl = lsl && L[q] == std::max<int64_t>(0, lo_abs - dq);
                }
                if (!heq) {
                    if (hca) fl |= kCausal;
                    else fit = false;
                }
                if (!leq) {
                    if (lsl) fl |= kSlide;
                    else fit = false;
                }
            }
            if (fit) {
                int64_t mnL = INT64_MAX, mxH = -1;
                for (uint32_t q = 0; q < Tq; ++q) {
                    mnL = std::min(mnL, L[q]);
                    mxH = std::max(mxH, H[q]);
                }
                subs.push_back(Sub{(uint32_t)(mnL / 16), (uint32_t)((mxH + 15) / 16), false, true, fl, lo_abs, hi_abs});
            } else {
                subs.push_back(Sub{(uint32_t)(hlo / 16), (uint32_t)((hhi + 15) / 16), true, false, 0, 0, 0});
            }
        }
    }
    if (subs.empty()) {                       // rule 8: no visible cell -> one empty chunk
        out.push_back(FaItem{q0, Tq, 0, 1, 0, 0, 0, 0});
        return TSRC_OK;
    }
    uint32_t n_total = 0;
    for (const Sub& s : subs) n_total += s.uhi - s.ulo;
    const uint32_t ncg = chunk_groups(in.C, in.pcap, E, in.D, n_total);
    if (ncg == 0) {
        *why = "FLASH_ATTN: the chunk size NCG is 0 for this PCAP / E / D";
        return TSRC_E_SHAPE;
    }
    std::vector<FaItem> list;
    for (const Sub& s : subs) {
        std::vector<uint32_t> cuts;
        for (uint64_t x = (uint64_t)s.ulo + ncg; x < s.uhi; x += ncg) cuts.push_back((uint32_t)x);
        if (s.multi && s.flags) {             // rule 5: no cut strictly inside a bound spread
            int64_t sp[2][2];
            uint32_t nsp = 0;
            if (s.flags & kCausal) {
                sp[nsp][0] = s.hi - (int64_t)(Tq - 1);
                sp[nsp][1] = s.hi;
                ++nsp;
            }
            if (s.flags & kSlide) {
                sp[nsp][0] = std::max<int64_t>(0, s.lo - (int64_t)(Tq - 1));
                sp[nsp][1] = s.lo;
                ++nsp;
            }
            for (int round = 0; round < 8; ++round) {
                bool changed = false;
                for (size_t i = 0; i < cuts.size(); ++i) {        // cuts added here are examined too
                    const int64_t X = 16 * (int64_t)cuts[i];
                    for (uint32_t t = 0; t < nsp; ++t) {
                        if (sp[t][0] < X && X < sp[t][1]) {
                            cuts[i] = (uint32_t)(sp[t][0] / 16);
                            cuts.push_back((uint32_t)((sp[t][1] + 15) / 16));
                            changed = true;
                            break;
                        }
                    }
                }
                std::sort(cuts.begin(), cuts.end());
                std::vector<uint32_t> kept;
                for (uint32_t c : cuts) {
                    if (c <= s.ulo || c >= s.uhi) continue;
                    if (!kept.empty() && kept.back() == c) continue;
                    kept.push_back(c);
                }
                cuts.swap(kept);
                if (!changed) break;
            }
        }
        uint32_t a = s.ulo;
        for (size_t i = 0; i <= cuts.size(); ++i) {
            const uint32_t b = i < cuts.size() ? cuts[i] : s.uhi;
            FaItem c{q0, Tq, 0, 0, 0, 0, 0, 0};
            if (!encode(s, Tq, L, H, a, b, c)) {
                *why = "FLASH_ATTN: the mask's runs admit no chunk encoding";
                return TSRC_E_SHAPE;
            }
            list.push_back(c);
            a = b;
        }
    }
    // rule 7: chunks holding a cell written in this launch run last, in their order
    for (int pass = 0; pass < 2; ++pass)
        for (const FaItem& c : list) {
            const uint64_t A = 16u * (uint64_t)c.u0, B = 16u * ((uint64_t)c.u0 + c.n);
            const bool nw = in.new_hi > in.new_lo && in.new_lo < B && in.new_hi > A;
            if ((int)nw == pass) out.push_back(c);
        }
    return TSRC_OK;
}

}  // namespace

int fa_plan(const FaPlanIn& in, FaPlanOut* po, FaItem** items, uint32_t* n_items, uint32_t** tile_items, const char** why) {
    *items = nullptr;
    *tile_items = nullptr;
    *n_items = 0;
    if (in.C == 0 || in.C > 16 || in.t_max == 0 || in.t_max > 8) {
        *why = "FLASH_ATTN: C must be 1..16 and T_MAX 1..8";
        return TSRC_E_SHAPE;
    }
    if (in.T == 0) {
        *why = "FLASH_ATTN: no query token";
        return TSRC_E_SHAPE;
    }
    if (!(in.D == 64 || in.D == 128 || in.D == 256 || in.D == 512) || in.n_head_kv == 0 || in.n_head % in.n_head_kv) {
        *why = "FLASH_ATTN: head_dim must be 64/128/256/512 and n_head a multiple of n_head_kv";
        return TSRC_E_SHAPE;
    }
    // E of the whole model (a shard of the KV heads plans as the single device does)
    const uint32_t plan_h = in.plan_n_head_kv ? in.plan_n_head_kv : in.n_head_kv;
    const uint32_t G = in.n_head / in.n_head_kv, E = plan_h * in.D;
    if (G == 0 || G > 64 || E / 64u > 511u) {
        *why = "FLASH_ATTN: G must be 1..64 and E / 64 at most 511";
        return TSRC_E_SHAPE;
    }
    if (in.k_max && (uint64_t)G * E > in.k_max) {
        *why = "FLASH_ATTN: G * E exceeds K_MAX";
        return TSRC_E_SHAPE;
    }
    const uint32_t GS0 = std::min(G, in.t_max), Tq0 = in.t_max / GS0;
    if (plan_h * GS0 * Tq0 > 128u || Tq0 * G * plan_h > 1024u) {
        *why = "FLASH_ATTN: a tile has more than 128 head rows or 1024 query rows";
        return TSRC_E_SHAPE;
    }
    if (chunk_groups(in.C, in.pcap, E, in.D, 1) == 0) {
        *why = "FLASH_ATTN: the chunk size NCG is 0 for this PCAP / E / D";
        return TSRC_E_SHAPE;
    }
    std::vector<Run> rows;
    const bool general = summarize(in.mask, in.mask_stride, in.n_kv, in.T, rows);
    std::vector<FaItem> list;
    std::vector<uint32_t> tiles;
    for (uint32_t q0 = 0; q0 < in.T; q0 += Tq0) {
        const uint32_t Tq = std::min(Tq0, in.T - q0);
        tiles.push_back((uint32_t)list.size());
        const int rc = plan_tile(in, E, general, rows.data() + q0, q0, Tq, list, why);
        if (rc != TSRC_OK) return rc;
    }
    tiles.push_back((uint32_t)list.size());
    po->Tq0 = Tq0;
    po->G = G;
    po->n_tiles = (uint32_t)tiles.size() - 1u;
    po->general = false;
    po->n_max_groups = 1;
    for (const FaItem& c : list) {
        po->n_max_groups = std::max(po->n_max_groups, c.n);
        po->general = po->general || c.general;
    }
    *items = new FaItem[list.size()];
    std::copy(list.begin(), list.end(), *items);
    *tile_items = new uint32_t[tiles.size()];
    std::copy(tiles.begin(), tiles.end(), *tile_items);
    *n_items = (uint32_t)list.size();
    return TSRC_OK;
}

void fa_plan_free(FaItem* items, uint32_t* tile_items) {
    delete[] items;
    delete[] tile_items;
}

}  // namespace tsrc
