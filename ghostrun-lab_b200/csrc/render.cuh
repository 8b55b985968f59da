// Warp-per-frame renderer for sm_100a: one warp draws one (env, frame) observation, 240x224 colour numbers (or
// their 6-bit packed form) plus 224 emphasis bytes, by replaying the frame log through FCEUmm's line renderer
// (the reference's batch_frame.cuh, third_party/nesle-extensions.patch:1246-1738, as called by
// rl/csrc/nes_machine.cuh:133-155 render_obs).
//
// The replay state (PPU address, scroll, control, palette, sprite lists, sprite-0 bookkeeping) is identical in all
// 32 lanes and advanced in lockstep; only the parallel parts are split:
//   * tile fetch: lane L fetches tile L of the line from the frame's nametable (staged in shared memory); the
//     pattern row comes from a 4-bit-per-pixel table ("sel" word: pixel k of the tile in bits 4k..4k+1) in shared
//     memory or, for banked / CHR-RAM boards, from the raw CHR bytes through a bit-spread table. Tiles 32-33 only
//     feed pixels right of the 240-pixel crop; they are fetched when a sprite-0 check reaches there or when an exact
//     line needs the shift registers;
//   * pixels: lane L draws pixels 8L..8L+7 from fetches L and L+1 (a funnel shift applies fine x); the palette
//     lookup is three byte permutes per four pixels;
//   * sprite evaluation: each lane holds OAM entries L and L+32 in registers for the frame; a ballot finds the
//     sprites on the next line and the first 8 in OAM order are fetched; lines without sprites skip it;
//   * sprite composition: per lane, bit-parallel over its 8 pixels;
//   * output: lanes 1..30 hold the 240-pixel crop; 8-byte stores, or 12-byte 6-bit packed groups per lane pair.
// Lines with frame-log writes landing inside the drawn part (mid-line splits) take the exact sequential tile loop
// (every lane runs it in lockstep) into a 256-byte shared line buffer.
#pragma once
#include "emulate.cuh"

namespace gr {

struct RSprites {   // per warp, shared memory: a sprite line (FetchSpriteData / RefreshSprites); its count is in
                    // the replay state (RState::nf / nd)
    u32 cw[8];      // colour nibbles of the 8 pixels left to right (flip applied), 0 = transparent
    u32 meta[8];    // palette attr (bits 0-1) | behind (bit 2) | x << 8
    u32 opq0;       // first fetched sprite: bit k = its pixel k (screen order) is opaque (sprite-0 hit data)
};

struct RWarp {      // per-warp shared scratch
    RSprites spr[2];     // fetched / drawn (double buffer)
    u32 pal[8];          // palette RAM of the replay (4 bytes per word)
    uint4 bgp;           // background sub-palettes 0-3 as drawn: colour 0 = backdrop | 0x40, & 0x3F (from pal)
    u32 chr[8];          // 1 KB CHR page per slot (paged boards)
    u32 lzchr[8];        // CHR pages of the line whose shift registers are kept lazily
    alignas(16) u8 nt[2048];  // the frame's nametable snapshot
    alignas(16) u8 px[256];   // exact-path line buffer
    u8 emph[224];
};

// Two-phase drawing of a frame without mid-line writes: a walk of the frame log (one lane per frame) records each
// line's replay state; the warp then draws the lines from the records with no per-line bookkeeping.
constexpr u32 kWalkVers = 4;   // palette / CHR-page versions a frame may use; more take the sequential path

struct FrameWalk {   // per frame, shared memory
    // line l: x = v | fine x << 15 | ctrl bits 3-5 << 18 | page map << 21;
    //         y = mask | palette version << 8 | CHR version << 12 | (mask & 0x10 at the line end) << 16 |
    //             palette version at the line end << 20
    uint2 rec[kObsY0 + kObsH];
    u32 pal[kWalkVers][8];       // palette RAM per version
    uint4 bgp[kWalkVers];        // background sub-palettes as drawn: colour 0 = backdrop, colours 1-3 | 0x40
    uint4 spal[kWalkVers];       // sprite sub-palettes & 0x3F
    u32 chr[kWalkVers][8];       // CHR pages per version
    u32 seq;                     // 1: the frame takes the sequential path (Renderer::draw)
    u32 split[8];                // bit l: line l was drawn exactly by the walk (a write inside its drawn part)
    alignas(16) u8 rows[4][256]; // draw_fast: the 4 lines of an iteration with sprites, byte x - 8 = screen x
};

struct RenderArgs {
    CartView cart;
    StateView st;
    u8* obs;             // [N, 4, 224, 240]
    u8* packed;          // [N, 4, 224, 180] 6-bit packed pictures, or nullptr
    u8* emph;            // [N, 4, 224]
    const u32* list;     // env list (restart pass), nullptr = all envs [e0, e0 + count)
    const u32* list_count;
    const u8* skip;      // envs to leave out (non-zero), nullptr = none
    u8* seqf;            // [N, 4]: 1 = the frame is left to the sequential renderer (k_render_seq)
    unsigned long long* stats;   // [2]: frames drawn by k_render_seq, lines drawn exactly by the walk (split lines)
    u32 e0, count;       // global env range of this launch (game slice)
    u32 frames;          // frames per env to draw (4)
    u32 chrx_smem;       // 1: the cart's pattern table is staged in shared memory (8 KB CHR ROM boards)
    u32 one;             // 1 (a run-time value: the kernels add disjoint bit fields as x * one + y, multiply-adds)
};

__device__ __forceinline__ u32 spread8(u32 b) {   // bit (7-k) of b -> bit 4k
    u32 r = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) r |= ((b >> (7 - k)) & 1u) << (4 * k);
    return r;
}

__device__ __forceinline__ u32 nib_reverse(u32 w) {   // nibble k -> nibble 7-k
    const u32 r = __byte_perm(w, 0, 0x0123);
    return ((r >> 4) & 0x0F0F0F0Fu) | ((r << 4) & 0xF0F0F0F0u);
}

__device__ __forceinline__ u32 nib_opaque8(u32 w) {   // bit k = nibble k has a colour
    u32 t = (w | (w >> 1)) & 0x11111111u;
    t = (t | (t >> 3)) & 0x03030303u;
    t = (t | (t >> 6)) & 0x000F000Fu;
    return (t | (t >> 12)) & 0xFFu;
}

// 4 pixels from 4 nibbles (c | attr << 2) through a 16-entry palette held as 4 words.
__device__ __forceinline__ u32 pal_lookup4(u32 sel16, u32 p0, u32 p1, u32 p2, u32 p3) {
    const u32 s = sel16 & 0x7777u;
    const u32 r1 = __byte_perm(p0, p1, s);
    const u32 r2 = __byte_perm(p2, p3, s);
    const u32 m = __byte_perm(0u, 0xFFFFFFFFu, (sel16 >> 1) & 0x4444u);   // 0xFF where attribute bit 1 is set
    return (r1 & ~m) | (r2 & m);
}

// prmt.b32 in its default mode (PTX ISA, prmt): a selector nibble with bit 3 set gives the sign bit of the byte its
// low 3 bits select, replicated over the target byte, so such a byte below 0x80 reads 0.
__device__ __forceinline__ u32 prmt_signed(u32 a, u32 b, u32 s) {
    u32 r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(s));
    return r;
}

// The same lookup for palette bytes below 0x80 in two permutes: (p0, p1) serve the nibbles whose attribute bit 1 is
// clear and read 0 where it is set; (p2, p3) take the nibbles with bit 3 flipped (sx = s ^ 0x8888), the other half.
// The halves have no bit in common, so they are joined by a multiply-add with `one` = 1 (a run-time value, so the
// compiler keeps the multiply): the integer multiply-add pipe has twice the integer logic pipe's rate and is idle here.
__device__ __forceinline__ u32 pal_lookup4s(u32 s, u32 sx, u32 p0, u32 p1, u32 p2, u32 p3, u32 one) {
    return prmt_signed(p2, p3, sx) * one + prmt_signed(p0, p1, s);
}

// nibble mask (4 nibbles, each 0 or 0xF, low 16 bits) -> byte mask
__device__ __forceinline__ u32 nib_to_bytes(u32 nm16) { return __byte_perm(0u, 0xFFFFFFFFu, nm16 & 0x4444u); }


// 4 colour numbers (bits 0-5 of each byte; bits 6-7 are ignored) -> their 24-bit 6-bit group in bits 0-23
// (rl/csrc/rlenv.cu:126-134 layout) with leftovers in bits 24-31, which the joins of groups into words leave out: two
// shift + merge steps. The right shifts are high halves of multiplies by m30 = 1 << 30 and m28 = 1 << 28 (run-time
// values, so the compiler keeps the multiplies): x >> k = (x * 2^(32-k)) >> 32 runs on the integer multiply-add pipe,
// which the renderer leaves mostly idle, instead of the integer logic pipe that bounds it.
__device__ __forceinline__ u32 pack_group6_loose(u32 w, u32 m30, u32 m28) {
    const u32 u = w ^ ((w ^ __umulhi(w, m30)) & 0x0FC00FC0u);   // c0 | c1 << 6 in bits 0-11, c2 | c3 << 6 in 16-27
    return u ^ ((u ^ __umulhi(u, m28)) & 0xFFFFF000u);           // bits 16-27 down to 12-23
}

// 4 colour numbers (bytes) -> one 24-bit 6-bit group (rl/csrc/rlenv.cu:126-134 layout)
__device__ __forceinline__ u32 pack_group6(u32 w) {
    return (w & 0x3Fu) | ((w >> 2) & 0xFC0u) | ((w >> 4) & 0x3F000u) | ((w >> 6) & 0xFC0000u);
}

struct RState {
    u32 v, t, x, ctrl, mask, mirroring;
    u32 sh0, sh1, at;    // tile shift registers (low 16 bits) and attribute latch
    u32 blurp, spork, hit, sphitx, sphitmask, hit_x;
    u32 fb;              // which of the two sprite buffers is `fetched`
    u32 fsame;           // 1: `fetched` holds what `drawn` holds (no fetch since the last copy), W.spr[fb ^ 1]
    u32 spal[4];         // sprite palette taken at RefreshSprites (& 0x3F)
    u32 lazy, lz_v, lz_ctrl, lz_mir;   // shift registers not yet materialised: fetches 32 / 33 of the line at lz_v
    u32 lz_saved;        // W.lzchr holds the lazy line's CHR pages (saved at the first CHR write after that line)
    u32 nf, nd;          // sprites in the fetched / drawn buffer
    u32 latch[2], creg[4];   // MMC2: the latches and CHR registers of the replay
    u32 cursor;
    int next_t;          // FCEUmm time of event `cursor`, INT_MAX past the last
};

template <u32 BOARD>
struct Renderer {
    const RenderArgs& A;
    const u32 lane;
    const u32* __restrict__ chrx;    // shared (or global) pattern table
    const u32* __restrict__ spread;  // shared 256-entry bit spread table
    RWarp& W;
    const u32* h;
    const u32* ev;
    u32 count;
    int kook;
    const u8* chr_ram;   // per-frame CHR-RAM snapshot, nullptr on CHR-ROM carts
    u32 spA, spB;        // OAM entries lane and lane + 32: y | tile << 8 | attr << 16 | x << 24
    RState s;
    int xs_line;         // the last line the walk drew exactly, -1 none; its final shift registers:
    u32 xs_sh0, xs_sh1, xs_at;

    __device__ Renderer(const RenderArgs& a, u32 ln, const u32* cx, const u32* sp, RWarp& w)
        : A(a), lane(ln), chrx(cx), spread(sp), W(w) {}

    __device__ __forceinline__ int ev_time(u32 i) const { return fceumm_time(ev[2 * i] & 0x1FFFFu, kook); }
    __device__ __forceinline__ int time_of(u32 i) const { return i < count ? ev_time(i) : 0x7FFFFFFF; }
    // apply event `cursor` and move on
    __device__ __forceinline__ void next_event(bool drawing) {
        apply(s.cursor, drawing);
        ++s.cursor;
        s.next_t = time_of(s.cursor);
    }
    // background sub-palette words for the fast line path (after the header and every palette write)
    __device__ __forceinline__ void make_bgp() {
        const u32 bd = (W.pal[0] & 0x3Fu) | 0x40u;
        W.bgp = make_uint4((W.pal[0] & 0x3F3F3F00u) | bd, (W.pal[1] & 0x3F3F3F00u) | bd,
                           (W.pal[2] & 0x3F3F3F00u) | bd, (W.pal[3] & 0x3F3F3F00u) | bd);
    }
    __device__ __forceinline__ u32 pal_byte(u32 i) const { return reinterpret_cast<const u8*>(W.pal)[i]; }
    // the CHR-RAM a presentation slot was frozen with (its own copy or the env's shared snapshot); CHR ROM: nullptr
    __device__ __forceinline__ const u8* slot_chr(u32 ge, u64 sl) const {
        if (A.cart.chr != nullptr || !A.st.snap_chr) return nullptr;
        if (A.st.chr_ref && A.st.chr_ref[sl]) return A.st.chr_shared + static_cast<u64>(ge) * kChrRamBytes;
        return A.st.snap_chr + sl * kChrRamBytes;
    }
    __device__ __forceinline__ static constexpr bool paged() { return board_paged(BOARD); }
    static constexpr bool kSplitLines = BOARD == kMmc3;   // the walk draws mid-line-write lines itself

    __device__ __forceinline__ u32 nt_rd(u32 mir, u32 addr) const {
        if constexpr (paged()) return W.nt[nt_off_map(mir, addr)];
        else return W.nt[nt_off_header(A.cart.arrangement, addr)];
    }
    __device__ __forceinline__ u32 chr_byte(const u32* pages, u32 addr) const {
        addr &= 0x1FFFu;
        if constexpr (paged()) {
            const u32 off = ((pages[addr >> 10] & A.cart.chr_page_mask) << 10) | (addr & 0x3FFu);
            return chr_ram ? chr_ram[off & 0x1FFFu] : __ldg(A.cart.chr + off);
        } else {
            return chr_ram ? chr_ram[addr] : __ldg(A.cart.chr + addr);   // CHR ROM is >= 8 KB: no wrap needed
        }
    }
    // colour nibbles of the pattern row at vadr (low-plane address)
    __device__ __forceinline__ u32 chr_sel(const u32* pages, u32 vadr) const {
        if constexpr (BOARD == kNrom || BOARD == kUxrom) {
            if (A.chrx_smem) {
                const u32 a = vadr & 0x1FFFu;
                return chrx[(a & 7u) * 512u + (a >> 4)];
            }
        }
        return spread[chr_byte(pages, vadr)] | (spread[chr_byte(pages, vadr + 8u)] << 1);
    }
    // One tile fetch at PPU address v: colour nibbles with the attribute in bits 2-3 of each nibble.
    __device__ __forceinline__ u32 fetch(u32 v, u32 ctrl, u32 mir, const u32* pages) const {
        const u32 base = 0x2000u | (v & 0x0C00u);
        const u32 tile = nt_rd(mir, base | (v & 0x3FFu));
        const u32 zz = v & 0x1Fu;
        const u32 ab = nt_rd(mir, base | 0x3C0u | (zz >> 2) | ((v & 0x380u) >> 4));
        const u32 attr = (ab >> ((zz & 2u) + ((v & 0x40u) >> 4))) & 3u;
        const u32 vadr = (tile << 4) + (((ctrl & 0x10u) << 8) | ((v >> 12) & 7u));
        return chr_sel(pages, vadr) | (attr * 0x44444444u);
    }

    // One line's background fetches with its uniform parts worked out once: the nametable page of the first and of
    // the wrapped tiles, the row, the pattern row; tile(c) = fetch c of the line (the c-th coarse-x increment of v).
    struct LineFetch {
        u32 cx0, base_a, base_b, row, arow, ashift, rowsel, vrow;
    };
    __device__ __forceinline__ u32 line_tile(const LineFetch& f, u32 c) const {
        const u32 cc = f.cx0 + c;
        const u32 col = cc & 31u;
        const u32 base = ((cc >> 5) & 1u) ? f.base_b : f.base_a;
        const u32 t = W.nt[base | f.row | col];
        const u32 ab = W.nt[base | f.arow | (col >> 2)];
        const u32 attr = (ab >> (f.ashift | (col & 2u))) & 3u;
        u32 sel;
        if constexpr (BOARD == kNrom || BOARD == kUxrom) {
            if (A.chrx_smem) sel = chrx[f.rowsel + t];
            else sel = chr_sel(W.chr, (t << 4) + f.vrow);
        } else {
            sel = chr_sel(W.chr, (t << 4) + f.vrow);
        }
        return sel | (attr * 0x44444444u);
    }
    __device__ __forceinline__ u32 nt_page(u32 which) const {   // CIRAM page (0/1) << 10 of nametable `which`
        if constexpr (paged()) return ((s.mirroring >> which) & 1u) << 10;
        else return (A.cart.arrangement == 1 ? (which >> 1) : which) << 10 & 0x400u;
    }
    __device__ __forceinline__ LineFetch line_fetch(u32 v) const {
        LineFetch f;
        f.cx0 = v & 0x1Fu;
        const u32 cy = (v >> 5) & 0x1Fu, which = (v >> 10) & 3u;
        f.base_a = nt_page(which);
        f.base_b = nt_page(which ^ 1u);
        f.row = cy << 5;
        f.arow = 0x3C0u | ((cy >> 2) << 3);
        f.ashift = (cy & 2u) << 1;
        const u32 fy = (v >> 12) & 7u;
        f.rowsel = fy * 512u + ((s.ctrl & 0x10u) << 4);
        f.vrow = ((s.ctrl & 0x10u) << 8) | fy;
        return f;
    }

    __device__ void apply(u32 i, bool drawing) {
        const u32 w1 = ev[2 * i + 1];
        const u32 value = w1 & 0xFFu, aux = (w1 >> 8) & 0xFFu;
        const u32 inc = (s.ctrl & 4u) ? 32u : 1u;
        switch (ev[2 * i] >> 24) {
            case kEvCtrl: s.ctrl = value; s.t = (s.t & 0xF3FFu) | ((value & 3u) << 10); break;
            case kEvMask: s.mask = value; break;
            case kEvScroll:
                if (aux == 0) { s.t = (s.t & 0xFFE0u) | (value >> 3); s.x = value & 7u; }
                else s.t = (s.t & 0x8C1Fu) | ((value & 0xF8u) << 2) | ((value & 7u) << 12);
                break;
            case kEvAddr:
                if (aux == 0) s.t = (s.t & 0x00FFu) | ((value & 0x3Fu) << 8);
                else { s.t = (s.t & 0xFF00u) | value; s.v = s.t; }
                break;
            case kEvDataWrite: s.v = (s.v + (aux + 1u) * inc) & 0x7FFFu; break;
            case kEvDataRead:
                if (drawing && (s.mask & 0x18u)) s.v = v_inc_y(s.v);
                else s.v = (s.v + inc) & 0x7FFFu;
                break;
            case kEvPalette:
                __syncwarp();
                if (lane == 0) {
                    reinterpret_cast<u8*>(W.pal)[aux & 31u] = static_cast<u8>(value);
                    make_bgp();
                }
                __syncwarp();
                s.v = (s.v + inc) & 0x7FFFu;
                break;
            case kEvChr:
                __syncwarp();
                if constexpr (paged()) {
                    if (s.lazy && !s.lz_saved) {   // the lazy line was fetched with the pages before this write
                        if (lane < 8) W.lzchr[lane] = W.chr[lane];
                        s.lz_saved = 1;
                        __syncwarp();
                    }
                }
                if (lane == 0) W.chr[aux & 7u] = value;
                __syncwarp();
                break;
            case kEvMirror: s.mirroring = value; break;
            case kEvMmc2:
                if constexpr (BOARD == kMmc2) {
                    if (aux < 4u) { s.creg[aux] = value; mmc2_select(aux >> 1); }
                    else if (aux == 6u || aux == 7u) { s.latch[aux - 6u] = value & 1u; mmc2_select(aux - 6u); }
                }
                break;
            default: break;
        }
    }

    // MMC2 (patch:1385-1402): a half's four 1 KB pages from the register its latch picks; a fetched pattern address
    // in $0FD0-$0FEF / $1FD0-$1FEF puts that half on its $FD or $FE bank. Warp-uniform arguments.
    __device__ __forceinline__ void mmc2_select(u32 half) {
        __syncwarp();
        if (lane < 4) W.chr[4 * (half & 1u) + lane] = (s.creg[(2 * half + (s.latch[half & 1u] & 1u)) & 3u] * 4 + lane) & 0xFFu;
        __syncwarp();
    }
    __device__ __forceinline__ void mmc2_hook(u32 addr) {
        const u32 high = (addr >> 8) & 0xFFu, low = addr & 0xF0u;
        if (high >= 0x20u || (high & 0x0Fu) != 0x0Fu || (low != 0xD0u && low != 0xE0u)) return;
        const u32 half = high >> 4;
        s.latch[half] = low == 0xE0u ? 1u : 0u;
        mmc2_select(half);
    }

    // MMC2, an event-free line drawn with rendering on: fetch c = lane through the pages its latch had then (the last
    // $FD / $FE tile among fetches 0..c-1, else the latch the line started with; all 34 fetches use one pattern table,
    // so one half), fetch 32 in c32; the shift registers after fetches 32 / 33 and the line's final latch are kept.
    __device__ __forceinline__ u32 mmc2_fast_fetch(u32 v0, u32& c32) {
        const LineFetch lf = line_fetch(v0);
        const u32 hb = (s.ctrl >> 4) & 1u, fy = (v0 >> 12) & 7u;
        auto at = [&](u32 c, u32& attr) {
            const u32 cc = lf.cx0 + c, col = cc & 31u;
            const u32 base = ((cc >> 5) & 1u) ? lf.base_b : lf.base_a;
            const u32 ab = W.nt[base | lf.arow | (col >> 2)];
            attr = (ab >> (lf.ashift | (col & 2u))) & 3u;
            return static_cast<u32>(W.nt[base | lf.row | col]);
        };
        auto nib = [&](u32 tile, u32 latch, u32 attr) {
            const u32 bank = s.creg[(2 * hb + (latch & 1u)) & 3u];
            const u32 off = (((bank * 4u + (tile >> 6)) & A.cart.chr_page_mask) << 10) | ((tile & 63u) << 4) | fy;
            return spread[__ldg(A.cart.chr + off)] | (spread[__ldg(A.cart.chr + off + 8u)] << 1) | (attr * 0x44444444u);
        };
        u32 a0, a32, a33;
        const u32 t = at(lane, a0), t32 = at(32, a32), t33 = at(33, a33);
        const u32 fm = __ballot_sync(0xFFFFFFFFu, t == 0xFDu || t == 0xFEu);
        const u32 fe = __ballot_sync(0xFFFFFFFFu, t == 0xFEu);
        const u32 lin = s.latch[hb];
        const u32 below = fm & ((1u << lane) - 1u);
        const u32 lc = below ? (fe >> (31 - __clz(below))) & 1u : lin;
        const u32 l32 = fm ? (fe >> (31 - __clz(fm))) & 1u : lin;
        const u32 l33 = (t32 == 0xFDu || t32 == 0xFEu) ? (t32 == 0xFEu ? 1u : 0u) : l32;
        const u32 lout = (t33 == 0xFDu || t33 == 0xFEu) ? (t33 == 0xFEu ? 1u : 0u) : l33;
        c32 = nib(t32, l32, a32);
        const u32 c33 = nib(t33, l33, a33);
        u32 lo32 = 0, hi32 = 0, lo33 = 0, hi33 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            lo32 |= ((c32 >> (4 * k)) & 1u) << (7 - k); hi32 |= ((c32 >> (4 * k + 1)) & 1u) << (7 - k);
            lo33 |= ((c33 >> (4 * k)) & 1u) << (7 - k); hi33 |= ((c33 >> (4 * k + 1)) & 1u) << (7 - k);
        }
        s.sh0 = (lo32 << 8) | lo33;
        s.sh1 = (hi32 << 8) | hi33;
        s.at = ((c32 >> 2) & 3u) | (((c33 >> 2) & 3u) << 2);
        const u32 ca = nib(t, lc, a0);
        if (lout != lin) { s.latch[hb] = lout; mmc2_select(hb); }
        return ca;
    }

    // The shift registers after the last fast line: its fetches 32 and 33.
    __device__ void materialize_shift() {
        if (!s.lazy) return;
        __syncwarp();
        const u32* pages = s.lz_saved ? W.lzchr : W.chr;
        const u32 c32 = fetch(v_inc_x_n(s.lz_v, 32), s.lz_ctrl, s.lz_mir, pages);
        const u32 c33 = fetch(v_inc_x_n(s.lz_v, 33), s.lz_ctrl, s.lz_mir, pages);
        u32 lo32 = 0, hi32 = 0, lo33 = 0, hi33 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            lo32 |= ((c32 >> (4 * k)) & 1u) << (7 - k); hi32 |= ((c32 >> (4 * k + 1)) & 1u) << (7 - k);
            lo33 |= ((c33 >> (4 * k)) & 1u) << (7 - k); hi33 |= ((c33 >> (4 * k + 1)) & 1u) << (7 - k);
        }
        s.sh0 = (lo32 << 8) | lo33;
        s.sh1 = (hi32 << 8) | hi33;
        s.at = ((c32 >> 2) & 3u) | (((c33 >> 2) & 3u) << 2);
        s.lazy = 0;
    }

    // ---- exact sequential path for a line with writes inside its drawn part (all lanes in lockstep)
    __device__ void exact_line(int l) {
        materialize_shift();
        const int start = l * 341 - 16;
        int firsttile = 0, outpos = 0;
        bool tofix = true;
        for (int q = lane; q < 256; q += 32) W.px[q] = 0xFF;
        __syncwarp();
        auto tiles = [&](int last) {
            const int first = firsttile;
            const u32 bd = (pal_byte(0) & 0x3Fu) | 0x40u;
            if (!(s.mask & 0x18u)) {
                for (int p = outpos + static_cast<int>(lane); p < outpos + 8 * (last - first) && p < 256; p += 32) W.px[p] = static_cast<u8>(bd);
                outpos += 8 * (last - first);
                firsttile = last;
                __syncwarp();
                return;
            }
            for (int tile = first; tile < last; ++tile) {
                if (tile >= 2) {
                    if (outpos < 256 && lane < 8) {
                        const u32 k = lane;
                        const u32 lo = (s.sh0 >> (8 - s.x)) & 0xFFu, hi = (s.sh1 >> (8 - s.x)) & 0xFFu;
                        const u32 c = ((lo >> (7 - k)) & 1u) | (((hi >> (7 - k)) & 1u) << 1);
                        const u32 at = (k + s.x) < 8 ? (s.at & 3u) : ((s.at >> 2) & 3u);
                        W.px[outpos + k] = static_cast<u8>(c == 0 ? bd : (pal_byte(at * 4 + c) & 0x3Fu));
                    }
                    outpos += 8;
                }
                const u32 v = s.v;
                const u32 base = 0x2000u | (v & 0x0C00u);
                const u32 tile_i = nt_rd(s.mirroring, base | (v & 0x3FFu));
                const u32 zz = v & 0x1Fu;
                const u32 ab = nt_rd(s.mirroring, base | 0x3C0u | (zz >> 2) | ((v & 0x380u) >> 4));
                const u32 attr = (ab >> ((zz & 2u) + ((v & 0x40u) >> 4))) & 3u;
                const u32 vadr = (tile_i << 4) + (((s.ctrl & 0x10u) << 8) | ((v >> 12) & 7u));
                const u32 p0 = chr_byte(W.chr, vadr), p1 = chr_byte(W.chr, vadr + 8u);   // both before the hook
                if constexpr (BOARD == kMmc2) mmc2_hook(vadr);
                s.at = ((s.at >> 2) | (attr << 2)) & 0xFu;
                s.sh0 = ((s.sh0 << 8) | p0) & 0xFFFFu;
                s.sh1 = ((s.sh1 << 8) | p1) & 0xFFFFu;
                s.v = v_inc_x(v);
            }
            __syncwarp();
            if (first <= 2 && 2 < last && !(s.mask & 0x02u)) { if (lane < 8) W.px[lane] = static_cast<u8>(bd); }
            if (!(s.mask & 0x08u)) {
                int ts = first - 2, tc = last - first;
                if (ts < 0) { tc += ts; ts = 0; }
                for (int p = ts * 8 + static_cast<int>(lane); p < (ts + tc) * 8 && p < 256; p += 32) W.px[p] = static_cast<u8>(bd);
            }
            firsttile = last;
            __syncwarp();
        };
        auto check = [&](int pp) {
            if (s.sphitx == 0x100u) return;
            for (int xx = static_cast<int>(s.sphitx); xx < static_cast<int>(s.sphitx) + 8 && xx < pp - 16 && xx < 255; ++xx) {
                if (((s.sphitmask >> (xx - static_cast<int>(s.sphitx))) & 1u) && !(W.px[xx] & 0x40u)) {
                    s.hit = 1; s.hit_x = static_cast<u32>(xx); s.sphitx = 0x100u; return;
                }
            }
        };
        auto update = [&](int pp) {
            int last = pp >> 3;
            if (s.sphitx != 0x100u && static_cast<int>(s.sphitx) < pp - 16 && !(static_cast<int>(s.sphitx) < (last - 2) * 8)) ++last;
            if (last > 34) last = 34;
            if (last <= firsttile) return;
            tiles(last);
            if (pp >= 268 && tofix) { if (s.mask & 0x18u) s.v = v_inc_y(s.v); tofix = false; }
            check(pp);
        };
        while (s.next_t < start + 272) {
            const u32 kind = ev[2 * s.cursor] >> 24;
            if (kind != kEvDataWrite && kind != kEvPalette)
                update(s.next_t + 3 * static_cast<int>((ev[2 * s.cursor] >> 17) & 0xFu) - start);
            next_event(true);
        }
        update(272);
        if (tofix) { if (s.mask & 0x18u) s.v = v_inc_y(s.v); tofix = false; }
        check(272);
        __syncwarp();
    }

    // ---- end of line: sprite fetch for line l + 1, Fixit2, RefreshSprites (patch:1652-1711)
    __device__ __forceinline__ void end_of_line(int l) {
        const int start = l * 341 - 16;
        s.sphitx = 0x100u;
        if (s.mask & 0x18u) {
            s.fsame = 0;
            RSprites& f = W.spr[s.fb];
            const u32 c = s.ctrl;
            const u32 hgt = (c & 0x20u) ? 16u : 8u;
            const bool in0 = static_cast<u32>(l - static_cast<int>(spA & 0xFFu)) < hgt;
            const bool in1 = static_cast<u32>(l - static_cast<int>(spB & 0xFFu)) < hgt;
            const u32 b0 = __ballot_sync(0xFFFFFFFFu, in0), b1 = __ballot_sync(0xFFFFFFFFu, in1);
            s.blurp = b0 & 1u;
            u32 n = 0;
            if constexpr (BOARD == kMmc2) {
                // in OAM order, each through the pages the previous fetches' hooks left
                if (b0 | b1) {
                    __syncwarp();
                    const u32 vofs = ((c & 0x08u) && !(c & 0x20u)) ? 0x1000u : 0u;
                    for (int half = 0; half < 2; ++half) {
                        for (u32 m = half ? b1 : b0; m && n < 8; m &= m - 1) {
                            const u32 sp = __shfl_sync(0xFFFFFFFFu, half ? spB : spA, __ffs(m) - 1);
                            const u32 tile = (sp >> 8) & 0xFFu, attr = (sp >> 16) & 0xFFu, xx = sp >> 24;
                            const u32 t = static_cast<u32>(l - static_cast<int>(sp & 0xFFu));
                            u32 vadr = hgt == 16u ? ((tile & 1u) << 12) + ((tile & 0xFEu) << 4) : (tile << 4) + vofs;
                            if (attr & 0x80u) { vadr += 7u; vadr -= t; vadr += (c & 0x20u) >> 1; vadr -= t & 8u; }
                            else { vadr += t; vadr += t & 8u; }
                            vadr &= 0x1FFFu;
                            u32 cw = chr_sel(W.chr, vadr);
                            if (attr & 0x40u) cw = nib_reverse(cw);
                            if (lane == 0) {
                                f.cw[n] = cw;
                                f.meta[n] = (attr & 3u) | ((attr & 0x20u) ? 4u : 0u) | (xx << 8);
                                if (n == 0) f.opq0 = nib_opaque8(cw);
                            }
                            mmc2_hook(vadr);
                            ++n;
                        }
                    }
                    __syncwarp();
                }
            } else if (b0 | b1) {
                __syncwarp();   // the previous line's readers of this buffer are done
                const u32 vofs = ((c & 0x08u) && !(c & 0x20u)) ? 0x1000u : 0u;
                const u32 lt = (1u << lane) - 1u;
                const u32 r0 = __popc(b0 & lt), r1 = __popc(b0) + __popc(b1 & lt);
                n = min(__popc(b0) + __popc(b1), 8);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const bool in = half ? in1 : in0;
                    const u32 r = half ? r1 : r0;
                    if (in && r < 8) {
                        const u32 sp = half ? spB : spA;
                        const u32 tile = (sp >> 8) & 0xFFu, attr = (sp >> 16) & 0xFFu, xx = sp >> 24;
                        const u32 t = static_cast<u32>(l - static_cast<int>(sp & 0xFFu));
                        u32 vadr = hgt == 16u ? ((tile & 1u) << 12) + ((tile & 0xFEu) << 4) : (tile << 4) + vofs;
                        if (attr & 0x80u) { vadr += 7u; vadr -= t; vadr += (c & 0x20u) >> 1; vadr -= t & 8u; }
                        else { vadr += t; vadr += t & 8u; }
                        u32 cw = chr_sel(W.chr, vadr & 0x1FFFu);
                        if (attr & 0x40u) cw = nib_reverse(cw);
                        f.cw[r] = cw;
                        f.meta[r] = (attr & 3u) | ((attr & 0x20u) ? 4u : 0u) | (xx << 8);
                        if (r == 0) f.opq0 = nib_opaque8(cw);
                    }
                }
                __syncwarp();
            }
            s.nf = n;
        }
        while (s.next_t < start + 278) next_event(true);
        if (s.mask & 0x18u) s.v = (s.v & 0xFBE0u) | (s.t & 0x041Fu);
        while (s.next_t < start + 341) next_event(true);
        if (s.mask & 0x10u) {
            s.spork = 0;
            // FCEUmm keeps one fetch buffer and copies it to the drawn one: without a fetch on this line (rendering
            // off at its end) the copy repeats the last fetch, which the drawn buffer already holds
            const bool same = s.fsame != 0;
            const RSprites& f = W.spr[same ? s.fb ^ 1u : s.fb];
            if ((same ? s.nd : s.nf) != 0) {
                if (!same) {
                    s.fb ^= 1u;    // drawn = fetched (the other buffer becomes the next fetch target)
                    const u32 t = s.nd;
                    s.nd = s.nf;
                    s.nf = t;
                    s.fsame = 1;
                }
                for (int q = 0; q < 4; ++q) s.spal[q] = W.pal[4 + q] & 0x3F3F3F3Fu;
                if (s.blurp && !s.hit && f.opq0) {
                    s.sphitx = f.meta[0] >> 8;
                    s.sphitmask = f.opq0;
                }
                s.spork = 1;
            }
        }
    }

    // ================================================================ two-phase path
    // ---- phase 1: replay the frame log's register state line by line (the same order of event application, v
    // increments and line ends as draw / end_of_line) and record it; pixels, sprites and sprite-0 bookkeeping are left
    // to phase 2 (sprite-0 state only changes what a mid-line write sees, and such frames take the sequential path).
    struct Walk {
        u32 ctrl, mask, x, v, t, mir, pv, cv, cursor, count, seq;
        bool pused, cused;
        int kook, next_t;
        const u32* ev;
    };
    __device__ __forceinline__ int walk_time(const Walk& w, u32 i) const {
        return i < w.count ? fceumm_time(w.ev[2 * i] & 0x1FFFFu, w.kook) : 0x7FFFFFFF;
    }
    __device__ static void derive(FrameWalk& F, u32 pv) {
        const u32* p = F.pal[pv];
        const u32 bd = p[0] & 0x3Fu;   // colours 1-3 carry bit 6 (opaque background, for sprite priority)
        F.bgp[pv] = make_uint4((p[0] & 0x3F3F3F00u) | 0x40404000u | bd, (p[1] & 0x3F3F3F00u) | 0x40404000u | bd,
                               (p[2] & 0x3F3F3F00u) | 0x40404000u | bd, (p[3] & 0x3F3F3F00u) | 0x40404000u | bd);
        F.spal[pv] = make_uint4(p[4] & 0x3F3F3F3Fu, p[5] & 0x3F3F3F3Fu, p[6] & 0x3F3F3F3Fu, p[7] & 0x3F3F3F3Fu);
    }
    __device__ void walk_apply(Walk& w, FrameWalk& F, bool drawing) const {
        const u32 w0 = w.ev[2 * w.cursor], w1 = w.ev[2 * w.cursor + 1];
        const u32 value = w1 & 0xFFu, aux = (w1 >> 8) & 0xFFu;
        const u32 inc = (w.ctrl & 4u) ? 32u : 1u;
        switch (w0 >> 24) {
            case kEvCtrl: w.ctrl = value; w.t = (w.t & 0xF3FFu) | ((value & 3u) << 10); break;
            case kEvMask: w.mask = value; break;
            case kEvScroll:
                if (aux == 0) { w.t = (w.t & 0xFFE0u) | (value >> 3); w.x = value & 7u; }
                else w.t = (w.t & 0x8C1Fu) | ((value & 0xF8u) << 2) | ((value & 7u) << 12);
                break;
            case kEvAddr:
                if (aux == 0) w.t = (w.t & 0x00FFu) | ((value & 0x3Fu) << 8);
                else { w.t = (w.t & 0xFF00u) | value; w.v = w.t; }
                break;
            case kEvDataWrite: w.v = (w.v + (aux + 1u) * inc) & 0x7FFFu; break;
            case kEvDataRead:
                if (drawing && (w.mask & 0x18u)) w.v = v_inc_y(w.v);
                else w.v = (w.v + inc) & 0x7FFFu;
                break;
            case kEvPalette:
                if (w.pused) {   // the current version is drawn with: the write starts a new one
                    if (w.pv + 1 >= kWalkVers) { w.seq = 1; break; }
                    for (int k = 0; k < 8; ++k) F.pal[w.pv + 1][k] = F.pal[w.pv][k];
                    ++w.pv;
                    w.pused = false;
                }
                reinterpret_cast<u8*>(F.pal[w.pv])[aux & 31u] = static_cast<u8>(value);
                w.v = (w.v + inc) & 0x7FFFu;
                break;
            case kEvChr:
                if (w.cused) {
                    if (w.cv + 1 >= kWalkVers) { w.seq = 1; break; }
                    for (int k = 0; k < 8; ++k) F.chr[w.cv + 1][k] = F.chr[w.cv][k];
                    ++w.cv;
                    w.cused = false;
                }
                F.chr[w.cv][aux & 7u] = value;
                break;
            case kEvMirror: w.mir = value; break;
            default: break;
        }
        ++w.cursor;
        w.next_t = walk_time(w, w.cursor);
    }
    // The header state, the frame's first tables and the events before the first line (group leader).
    __device__ void walk_begin(u32 ge, u32 f, FrameWalk& F, Walk& w) const {
        const u64 sl = static_cast<u64>(ge) * 4 + f;
        const u32* hh = A.st.log + (static_cast<u64>(ge) * kLogBanks + A.st.slot_bank[sl]) * kLogBankWords;
        w.ev = hh + kLogHdr;
        w.count = min(hh[0] & ~kLogOverflow, kLogEv);
        w.kook = (hh[15] & kLogKook) ? 1 : 0;
        w.ctrl = hh[1] & 0xFFu; w.mask = (hh[1] >> 8) & 0xFFu; w.x = (hh[1] >> 16) & 7u;
        w.v = hh[2] & 0x7FFFu; w.t = (hh[2] >> 16) & 0x7FFFu;
        w.mir = hh[5] & 0xFu;
        for (int k = 0; k < 8; ++k) {
            F.pal[0][k] = hh[7 + k];
            F.chr[0][k] = (hh[3 + (k >> 2)] >> ((k & 3) * 8)) & 0xFFu;
        }
        w.pv = 0; w.cv = 0; w.pused = false; w.cused = false; w.seq = 0;
        w.cursor = 0;
        w.next_t = walk_time(w, 0);
        while (w.next_t < -16 && !w.seq) walk_apply(w, F, false);
        if (w.mask & 0x18u) w.v = w.t;
    }
    // Line l with its events (group leader): the line-by-line replay order of draw / end_of_line.
    __device__ void walk_line(Walk& w, FrameWalk& F, int l) const {
        const int start = l * 341 - 16;
        if (w.next_t < start + 272) { w.seq = 1; return; }   // a write inside the drawn part of the line
        if (!w.pused) { derive(F, w.pv); w.pused = true; }
        w.cused = true;
        const u32 rx = w.v | (w.x << 15) | (((w.ctrl >> 3) & 7u) << 18) | ((w.mir & 0xFu) << 21);
        const u32 ry = w.mask | (w.pv << 8) | (w.cv << 12);
        const u32 fetch_mask = w.mask;
        if (w.mask & 0x18u) w.v = v_inc_y(v_inc_x_n(w.v, 34));
        while (w.next_t < start + 278 && !w.seq) walk_apply(w, F, true);
        if (w.mask & 0x18u) w.v = (w.v & 0xFBE0u) | (w.t & 0x041Fu);
        while (w.next_t < start + 341 && !w.seq) walk_apply(w, F, true);
        if (!w.pused) { derive(F, w.pv); w.pused = true; }
        // sprites switched on during the hblank of a line drawn with rendering off would show an older line's
        // sprite fetch (the buffer's count is stale): the sequential path keeps that
        if (!(fetch_mask & 0x18u) && (w.mask & 0x10u)) w.seq = 1;
        F.rec[l] = make_uint2(rx, ry | ((w.mask & 0x10u) ? (1u << 16) : 0u) | (w.pv << 20));
    }
    // The frame's nametable into shared memory, its OAM into registers (2 entries per lane), its CHR-RAM (all lanes).
    __device__ void load_frame(u32 ge, u32 f) {
        const u64 sl = static_cast<u64>(ge) * 4 + f;
        chr_ram = slot_chr(ge, sl);
        const uint4* ntg = reinterpret_cast<const uint4*>(A.st.snap_nt + sl * kNtBytes);
        uint4* nts = reinterpret_cast<uint4*>(W.nt);
        const uint4 q0 = ntg[lane], q1 = ntg[lane + 32], q2 = ntg[lane + 64], q3 = ntg[lane + 96];
        const u32* oamw = reinterpret_cast<const u32*>(A.st.snap_oam + sl * kOamBytes);
        spA = oamw[lane];
        spB = oamw[lane + 32];
        __syncwarp();
        nts[lane] = q0; nts[lane + 32] = q1; nts[lane + 64] = q2; nts[lane + 96] = q3;
        __syncwarp();
    }

    // Line l with a write inside its drawn part, drawn exactly by the whole warp during the walk (all lanes hold
    // the walk's state w): the sequential renderer's state at the start of line l from the walk (registers,
    // palette and CHR-page versions, the frame log cursor), the shift registers of the last line drawn with
    // rendering on (fetches 32 / 33 of that line, or the exact ones of a line drawn here), the sprites fetched at
    // the end of line l - 1; then exact_line, CopySprites, greyscale and the row's output as in draw. Returns with
    // the registers the line's writes left in s (the caller hands them back to the walk).
    __device__ void split_line(FrameWalk& F, const Walk& w, int l, u8* obs_out, bool pack6) {
        s.v = w.v; s.t = w.t; s.x = w.x; s.ctrl = w.ctrl; s.mask = w.mask; s.mirroring = w.mir;
        if (lane < 8) { W.pal[lane] = F.pal[w.pv][lane]; W.chr[lane] = F.chr[w.cv][lane]; }
        __syncwarp();
        if (lane == 0) make_bgp();
        ev = w.ev; count = w.count; kook = w.kook;
        s.cursor = w.cursor; s.next_t = w.next_t;
        s.lazy = 0; s.lz_saved = 0; s.sh0 = s.sh1 = s.at = 0;
        int j = l - 1;
        while (j >= 0 && !(F.rec[j].y & 0x18u)) --j;
        if (j >= 0 && j == xs_line) {
            s.sh0 = xs_sh0; s.sh1 = xs_sh1; s.at = xs_at;
        } else if (j >= 0) {
            const uint2 rj = F.rec[j];
            s.lazy = 1; s.lz_v = rj.x & 0x7FFFu; s.lz_ctrl = ((rj.x >> 18) & 7u) << 3; s.lz_mir = (rj.x >> 21) & 0xFu;
            if (lane < 8) W.lzchr[lane] = F.chr[(rj.y >> 12) & 3u][lane];
            s.lz_saved = 1;
        }
        // the sprites drawn on line l: fetched at the end of line l - 1 and refreshed there
        s.fb = 0; s.nd = 0; s.nf = 0; s.spork = 0; s.fsame = 0;
        if (l >= 1) {
            const uint2 re = F.rec[l - 1];
            if ((re.y & 0x18u) && (re.y & (1u << 16))) {
                const u32 c = ((re.x >> 18) & 7u) << 3;
                const u32 hgt = (c & 0x20u) ? 16u : 8u;
                const int e = l - 1;
                const bool in0 = static_cast<u32>(e - static_cast<int>(spA & 0xFFu)) < hgt;
                const bool in1 = static_cast<u32>(e - static_cast<int>(spB & 0xFFu)) < hgt;
                const u32 b0 = __ballot_sync(0xFFFFFFFFu, in0), b1 = __ballot_sync(0xFFFFFFFFu, in1);
                if (b0 | b1) {
                    RSprites& d = W.spr[1];
                    const u32* pages = F.chr[(re.y >> 12) & 3u];
                    const u32 vofs = ((c & 0x08u) && !(c & 0x20u)) ? 0x1000u : 0u;
                    const u32 lt = (1u << lane) - 1u;
                    const u32 r0 = __popc(b0 & lt), r1 = __popc(b0) + __popc(b1 & lt);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const bool in = half ? in1 : in0;
                        const u32 r = half ? r1 : r0;
                        if (in && r < 8) {
                            const u32 sp = half ? spB : spA;
                            const u32 tile = (sp >> 8) & 0xFFu, attr = (sp >> 16) & 0xFFu, xx = sp >> 24;
                            const u32 t = static_cast<u32>(e - static_cast<int>(sp & 0xFFu));
                            u32 vadr = hgt == 16u ? ((tile & 1u) << 12) + ((tile & 0xFEu) << 4) : (tile << 4) + vofs;
                            if (attr & 0x80u) { vadr += 7u; vadr -= t; vadr += (c & 0x20u) >> 1; vadr -= t & 8u; }
                            else { vadr += t; vadr += t & 8u; }
                            u32 cw = chr_sel(pages, vadr & 0x1FFFu);
                            if (attr & 0x40u) cw = nib_reverse(cw);
                            d.cw[r] = cw;
                            d.meta[r] = (attr & 3u) | ((attr & 0x20u) ? 4u : 0u) | (xx << 8);
                        }
                    }
                    s.nd = min(__popc(b0) + __popc(b1), 8);
                    s.spork = 1;
                }
                const uint4 sp4 = F.spal[(re.y >> 20) & 3u];
                s.spal[0] = sp4.x; s.spal[1] = sp4.y; s.spal[2] = sp4.z; s.spal[3] = sp4.w;
            }
        }
        s.sphitx = 0x100u; s.blurp = 0; s.hit = 0; s.sphitmask = 0; s.hit_x = 0;
        __syncwarp();
        exact_line(l);
        xs_line = l; xs_sh0 = s.sh0; xs_sh1 = s.sh1; xs_at = s.at;
        const uint2 q = reinterpret_cast<const uint2*>(W.px)[lane];
        u32 w0 = q.x, w1 = q.y;
        if ((s.mask & 0x10u) && s.spork) {   // CopySprites (patch:1615-1640)
            const RSprites& d = W.spr[1];
            u32 snib = 0, sany = 0, sbeh = 0;
            const int base = static_cast<int>(lane) * 8;
            for (int i = static_cast<int>(s.nd) - 1; i >= 0; --i) {
                const u32 meta = d.meta[i];
                const int dx = static_cast<int>(meta >> 8) - base;
                if (dx <= -8 || dx >= 8) continue;
                const u32 cw = d.cw[i];
                const u32 win = dx >= 0 ? (cw << (4 * dx)) : (cw >> (4 * -dx));
                const u32 om = ((win | (win >> 1)) & 0x11111111u) * 0xFu;
                const u32 pw = (meta & 3u) * 0x44444444u;
                snib = (snib & ~om) | ((win | pw) & om);
                sany |= om;
                sbeh = (meta & 4u) ? (sbeh | om) : (sbeh & ~om);
            }
            if (lane == 0 && !(s.mask & 0x04u)) sany = 0;
            if (sany) {
                const u32 c0 = pal_lookup4(snib, s.spal[0], s.spal[1], s.spal[2], s.spal[3]);
                const u32 c1 = pal_lookup4(snib >> 16, s.spal[0], s.spal[1], s.spal[2], s.spal[3]);
                const u32 any0 = nib_to_bytes(sany), any1 = nib_to_bytes(sany >> 16);
                const u32 beh0 = nib_to_bytes(sbeh), beh1 = nib_to_bytes(sbeh >> 16);
                const u32 tr0 = ((w0 & 0x40404040u) >> 6) * 0xFFu, tr1 = ((w1 & 0x40404040u) >> 6) * 0xFFu;
                const u32 use0 = any0 & (~beh0 | tr0), use1 = any1 & (~beh1 | tr1);
                w0 = (w0 & ~use0) | (c0 & use0);
                w1 = (w1 & ~use1) | (c1 & use1);
            }
        }
        const u32 keep = ((s.mask & 1u) && (s.mask & 0x18u)) ? 0x30303030u : 0x3F3F3F3Fu;
        w0 &= keep;
        w1 &= keep;
        if (l >= kObsY0) {
            const int y = l - kObsY0;
            if (!pack6) {
                if (lane >= 1 && lane <= 30)
                    reinterpret_cast<uint2*>(obs_out + static_cast<u64>(y) * kObsW)[lane - 1] = make_uint2(w0, w1);
            } else {
                const u32 g0 = pack_group6(w0), g1 = pack_group6(w1);
                const u32 n0 = __shfl_down_sync(0xFFFFFFFFu, g0, 1), n1 = __shfl_down_sync(0xFFFFFFFFu, g1, 1);
                if ((lane & 1u) && lane <= 29) {
                    u32* row = reinterpret_cast<u32*>(obs_out + static_cast<u64>(y) * (kObsW / 4 * 3)) + 3 * ((lane - 1) >> 1);
                    row[0] = g0 | (g1 << 24);
                    row[1] = (g1 >> 8) | (n0 << 16);
                    row[2] = (n0 >> 16) | (n1 << 8);
                }
            }
        }
        __syncwarp();
    }

    // ---- phase 1 for frame f of env ge (the whole warp): lane 0 replays the frame log's events; every stretch of
    // lines without events is recorded by the 32 lanes at once, v from the closed form above (the record of such a
    // line is its start state, unchanged through the line).
    __device__ void walk_frame(u32 ge, u32 f, FrameWalk& F, u8* obs_out, bool pack6) {
        constexpr int kLines = kObsY0 + kObsH;
        if constexpr (kSplitLines) {   // the exact lines need the frame's memories now; the others load in draw_fast
            load_frame(ge, f);
            if (lane < 8) F.split[lane] = 0;
            xs_line = -1;
        }
        Walk w;
        int l = 0;
        bool done = false;
        if (lane == 0) walk_begin(ge, f, F, w);
        for (;;) {
            int run = 0;
            u32 v = 0, xc = 0, ry = 0, th = 0, ren = 0, split = 0;
            if (lane == 0 && !done) {
                if (w.seq) {
                    done = true;
                } else {
                    if (!w.pused) { derive(F, w.pv); w.pused = true; }
                    w.cused = true;
                    // the next event is applied in line (next_t + 16) / 341: the lines before it have none
                    const int lev = w.next_t >= kLines * 341 ? kLines : (w.next_t + 16) / 341;
                    run = max(0, min(lev, kLines) - l);
                    v = w.v;
                    xc = (w.x << 15) | (((w.ctrl >> 3) & 7u) << 18) | ((w.mir & 0xFu) << 21);
                    ry = w.mask | (w.pv << 8) | (w.cv << 12) | ((w.mask & 0x10u) ? (1u << 16) : 0u) | (w.pv << 20);
                    th = w.t & 0x041Fu;
                    ren = (w.mask & 0x18u) ? 1u : 0u;
                    // after the stretch: a line with a write inside its drawn part is drawn here, exactly (MMC3,
                    // whose IRQ handlers split the screen; the other boards leave such frames to k_render_seq)
                    const int ls = l + run;
                    if constexpr (kSplitLines) {
                        split = (ls < kLines && w.next_t < ls * 341 - 16 + 272) ? 1u : 0u;
                        // FCEUmm draws one tile more before a mid-line write while sprite 0 is on the line and has
                        // not hit yet (replay_update's sphitx rule, patch:1593-1596), so where the write lands
                        // depends on the frame's sprite-0 state, which only the sequential renderer follows: a
                        // split line that sprite 0 may reach (fetched at the end of the line above, 8x16 at most;
                        // lane 0 holds OAM entry 0) sends the frame there
                        if (split && static_cast<u32>(ls - 1 - static_cast<int>(spA & 0xFFu)) < 16u) {
                            w.seq = 1;
                            split = 0;
                            run = 0;
                        }
                    }
                }
            }
            run = __shfl_sync(0xFFFFFFFFu, run, 0);
            const int l0 = __shfl_sync(0xFFFFFFFFu, l, 0);
            v = __shfl_sync(0xFFFFFFFFu, v, 0);
            xc = __shfl_sync(0xFFFFFFFFu, xc, 0);
            ry = __shfl_sync(0xFFFFFFFFu, ry, 0);
            th = __shfl_sync(0xFFFFFFFFu, th, 0);
            ren = __shfl_sync(0xFFFFFFFFu, ren, 0);
            if constexpr (kSplitLines) split = __shfl_sync(0xFFFFFFFFu, split, 0);
            for (int k = static_cast<int>(lane); k < run; k += 32)
                F.rec[l0 + k] = make_uint2(v_after_lines(v, static_cast<u32>(k), th, ren != 0) | xc, ry);
            if (lane == 0 && !done) {
                w.v = v_after_lines(w.v, static_cast<u32>(run), th, ren != 0);
                l += run;
            }
            if (kSplitLines && split) {
                const int ls = l0 + run;
                Walk wb;   // the leader's state, on every lane
                wb.ctrl = __shfl_sync(0xFFFFFFFFu, w.ctrl, 0); wb.mask = __shfl_sync(0xFFFFFFFFu, w.mask, 0);
                wb.x = __shfl_sync(0xFFFFFFFFu, w.x, 0); wb.v = __shfl_sync(0xFFFFFFFFu, w.v, 0);
                wb.t = __shfl_sync(0xFFFFFFFFu, w.t, 0); wb.mir = __shfl_sync(0xFFFFFFFFu, w.mir, 0);
                wb.pv = __shfl_sync(0xFFFFFFFFu, w.pv, 0); wb.cv = __shfl_sync(0xFFFFFFFFu, w.cv, 0);
                wb.cursor = __shfl_sync(0xFFFFFFFFu, w.cursor, 0); wb.count = __shfl_sync(0xFFFFFFFFu, w.count, 0);
                wb.kook = __shfl_sync(0xFFFFFFFFu, w.kook, 0); wb.next_t = __shfl_sync(0xFFFFFFFFu, w.next_t, 0);
                wb.ev = reinterpret_cast<const u32*>(__shfl_sync(0xFFFFFFFFu, reinterpret_cast<unsigned long long>(w.ev), 0));
                __syncwarp();   // the leader's derive of this line's palette version is visible
                split_line(F, wb, ls, obs_out, pack6);
                if (lane == 0) atomicAdd(A.stats + 1, 1ull);
                if (lane == 0) {
                    // the line's writes into the walk's copy-on-write tables; the exact registers replace the walk's
                    while (w.cursor < s.cursor && !w.seq) walk_apply(w, F, true);
                    w.v = s.v; w.t = s.t; w.x = s.x; w.ctrl = s.ctrl; w.mask = s.mask; w.mir = s.mirroring;
                    const int start = ls * 341 - 16;
                    const u32 rx = w.v | (w.x << 15) | (((w.ctrl >> 3) & 7u) << 18) | ((w.mir & 0xFu) << 21);
                    const u32 ryl = w.mask | (w.pv << 8) | (w.cv << 12);
                    const u32 fetch_mask = w.mask;
                    while (w.next_t < start + 278 && !w.seq) walk_apply(w, F, true);
                    if (w.mask & 0x18u) w.v = (w.v & 0xFBE0u) | (w.t & 0x041Fu);
                    while (w.next_t < start + 341 && !w.seq) walk_apply(w, F, true);
                    if (!w.pused) { derive(F, w.pv); w.pused = true; }
                    if (!(fetch_mask & 0x18u) && (w.mask & 0x10u)) w.seq = 1;
                    F.rec[ls] = make_uint2(rx, ryl | ((w.mask & 0x10u) ? (1u << 16) : 0u) | (w.pv << 20));
                    F.split[ls >> 5] |= 1u << (ls & 31);
                    l = ls + 1;
                }
            } else if (lane == 0 && !done) {
                if (l < kLines) walk_line(w, F, l++);
            }
            if (lane == 0 && !done && (l >= kLines || w.seq)) done = true;
            if (__shfl_sync(0xFFFFFFFFu, done ? 1u : 0u, 0) != 0u) break;
        }
        if (lane == 0) F.seq = w.seq;
        __syncwarp();
    }

    // One line's background fetch from a record (v, control, page map given).
    __device__ __forceinline__ LineFetch line_fetch_at(u32 v, u32 ctrl, u32 mir) const {
        LineFetch f;
        f.cx0 = v & 0x1Fu;
        const u32 cy = (v >> 5) & 0x1Fu, which = (v >> 10) & 3u;
        if constexpr (paged()) {
            f.base_a = ((mir >> which) & 1u) << 10;
            f.base_b = ((mir >> (which ^ 1u)) & 1u) << 10;
        } else {
            f.base_a = nt_page(which);
            f.base_b = nt_page(which ^ 1u);
        }
        f.row = cy << 5;
        f.arow = 0x3C0u | ((cy >> 2) << 3);
        f.ashift = (cy & 2u) << 1;
        const u32 fy = (v >> 12) & 7u;
        f.rowsel = fy * 512u + ((ctrl & 0x10u) << 4);
        f.vrow = ((ctrl & 0x10u) << 8) | fy;
        return f;
    }
    // Fetch c of a line in two parts: the nametable's tile t and attribute (the same for the 8 lines of a tile row; the
    // attribute as aw = attr * 0x44444444, its bits 2-3 in every nibble), then the pattern row of this line as colour
    // nibbles with the attribute added (disjoint bits: one multiply-add with `one` = 1).
    __device__ __forceinline__ void line_tile_ta(const LineFetch& f, u32 c, u32& t, u32& aw) const {
        const u32 cc = f.cx0 + c;
        const u32 col = cc & 31u;
        const u32 base = ((cc >> 5) & 1u) ? f.base_b : f.base_a;
        t = W.nt[base | f.row | col];
        const u32 ab = W.nt[base | f.arow | (col >> 2)];
        aw = ((ab >> (f.ashift | (col & 2u))) & 3u) * 0x44444444u;
    }
    __device__ __forceinline__ u32 line_tile_sel(u32 rowsel, u32 vrow, u32 t, u32 aw, const u32* pages, u32 one) const {
        u32 sel;
        if constexpr (BOARD == kNrom || BOARD == kUxrom) {
            if (A.chrx_smem) sel = chrx[rowsel + t];
            else sel = chr_sel(pages, (t << 4) + vrow);
        } else {
            sel = chr_sel(pages, (t << 4) + vrow);
        }
        return sel * one + aw;
    }

    // ---- phase 2 (the whole warp): draw frame f of env ge from its walk, 4 lines at a time: lane group g = lane / 8
    // draws line l0 + g, lane j = lane % 8 its crop pixels 32j..32j+31 (screen x 8+32j..): fetches 4j+1..4j+5.
    // The lines are independent given the records: the sprites drawn on line l are those fetched at the end of line
    // l - 1 (FetchSpriteData with line l - 1's control, CHR pages and OAM) when line l - 1 fetched (rendering on)
    // and the refresh at its end had sprites on (which is line l's mask); the walk sends the one case where an older
    // fetch would show to the sequential path. Crop x starts at 8, so the left-column clips never show.
    __device__ void draw_fast(u32 ge, u32 f, FrameWalk& F, u8* obs_out, u8* emph_out, bool pack6) {
        if constexpr (!kSplitLines) load_frame(ge, f);   // (boards with exact lines staged it in walk_frame)
        const u32 g = lane >> 3, j = lane & 7u;
        const u32 lt = (1u << lane) - 1u;
        // Lines that can show a sprite: one at y is found by the evaluation at the end of lines y..y+h-1 (height h) and
        // drawn on lines y+1..y+h. A superset; iterations whose 4 lines have none skip the sprite work.
        u32* may = reinterpret_cast<u32*>(W.emph);   // 8 words: bit l of the 256-line mask
        u8* vis = W.emph + 32;                       // OAM indices of the sprites that can show, in OAM order
        u32 nv;
        {
            // 8x16 sprites on any line of the frame (control bit 5 in the records): 16 lines per sprite, else 8
            u32 tall = 0;
            for (u32 l = lane; l < static_cast<u32>(kObsY0 + kObsH); l += 32) tall |= F.rec[l].x;
            const int extra = __any_sync(0xFFFFFFFFu, (tall >> 20) & 1u) ? 15 : 7;
            auto span = [extra](u32 sp, u32 base) -> u32 {
                const int lo = static_cast<int>(sp & 0xFFu) + 1 - static_cast<int>(base);
                const int hi = lo + extra;
                if (hi < 0 || lo > 31) return 0u;
                const u32 a = lo < 0 ? 0u : static_cast<u32>(lo), b = hi > 31 ? 31u : static_cast<u32>(hi);
                return (0xFFFFFFFFu >> (31u - b)) & (0xFFFFFFFFu << a);
            };
#pragma unroll
            for (u32 b = 0; b < 8; ++b) {
                const u32 m = __reduce_or_sync(0xFFFFFFFFu, span(spA, 32u * b) | span(spB, 32u * b));
                if (lane == 0) may[b] = m;
            }
            // a sprite at y is evaluated on lines y..y+15 at most; the evaluations that draw are on lines 7..230
            const bool va = (spA & 0xFFu) <= 230u, vb = (spB & 0xFFu) <= 230u;
            const u32 ba = __ballot_sync(0xFFFFFFFFu, va), bb = __ballot_sync(0xFFFFFFFFu, vb);
            if (va) vis[__popc(ba & lt)] = static_cast<u8>(lane);
            if (vb) vis[__popc(ba) + __popc(bb & lt)] = static_cast<u8>(lane + 32u);
            nv = __popc(ba) + __popc(bb);
            __syncwarp();
        }
        u32 key_prev = 0xFFFFFFFFu;   // this lane's cached tile row: tiles t0-t3, attributes aw0-aw3
        u32 t0 = 0, t1 = 0, t2 = 0, t3 = 0, aw0 = 0, aw1 = 0, aw2 = 0, aw3 = 0;
        const u32 one = A.one, m16 = one << 16, m28 = one << 28, m30 = one << 30;   // see pack_group6_loose
        for (int l0 = kObsY0; l0 < kObsY0 + kObsH; l0 += 4) {
            const bool any = ((may[l0 >> 5] >> (l0 & 31)) & 0xFu) != 0;   // warp-uniform
            // ---- background of line l (this lane group's), 32 pixels per lane
            const int l = l0 + static_cast<int>(g);
            const uint2 r = F.rec[l];
            const u32 mask = r.y & 0xFFu;
            const uint4 P = F.bgp[(r.y >> 8) & 3u];
            const u32 bdw = (P.x & 0xFFu) * 0x01010101u;
            u32 s0 = 0, s1 = 0, s2 = 0, s3 = 0;   // pixel nibbles (colour | attribute << 2), 8 per word
            const bool bg = (mask & 0x08u) != 0;
            // the tile row of the line (coarse x / y, nametable, page map): unchanged on every lane since the
            // iteration before (lines without background keep theirs) -> this lane's tiles and attributes are cached
            const u32 key = bg ? (r.x & 0x0FFFu) | (((r.x >> 21) & 0xFu) << 12) : key_prev;
            const bool fresh = __any_sync(0xFFFFFFFFu, key != key_prev);
            key_prev = key;
            u32 c0 = 0, c1 = 0, c2 = 0, c3 = 0;   // this lane's 4 fetches (0 where the background is off)
            if (bg) {
                const u32 ctrl = ((r.x >> 18) & 7u) << 3;
                const u32* pages = F.chr[(r.y >> 12) & 3u];
                if (fresh) {   // the tile row's nametable and attribute bytes
                    const LineFetch lf = line_fetch_at(r.x & 0x7FFFu, ctrl, (r.x >> 21) & 0xFu);
                    line_tile_ta(lf, 4 * j + 1, t0, aw0); line_tile_ta(lf, 4 * j + 2, t1, aw1);
                    line_tile_ta(lf, 4 * j + 3, t2, aw2); line_tile_ta(lf, 4 * j + 4, t3, aw3);
                }
                // this line's pattern row: fine y and the background pattern table
                const u32 fy = (r.x >> 12) & 7u;
                const u32 rowsel = fy * 512u + ((ctrl & 0x10u) << 4), vrow = ((ctrl & 0x10u) << 8) | fy;
                c0 = line_tile_sel(rowsel, vrow, t0, aw0, pages, one); c1 = line_tile_sel(rowsel, vrow, t1, aw1, pages, one);
                c2 = line_tile_sel(rowsel, vrow, t2, aw2, pages, one); c3 = line_tile_sel(rowsel, vrow, t3, aw3, pages, one);
            }
            // fetch 4j + 5 is the next lane's first (a full-warp shuffle, outside the per-line branch); lane 7's last
            // 16 pixels (screen x 248-263) are not drawn
            const u32 c4 = __shfl_down_sync(0xFFFFFFFFu, c0, 1);
            if (bg) {
                const u32 x4 = 4u * ((r.x >> 15) & 7u);
                s0 = __funnelshift_r(c0, c1, x4); s1 = __funnelshift_r(c1, c2, x4);
                s2 = __funnelshift_r(c2, c3, x4); s3 = __funnelshift_r(c3, c4, x4);
            }
            // colour bytes, 4 pixels per word: bits 0-5 the colour, bit 6 set where the background colour is not 0
            u32 px[8];
            if (bg) {
                const u32 x0 = s0 ^ 0x88888888u, x1 = s1 ^ 0x88888888u, x2 = s2 ^ 0x88888888u, x3 = s3 ^ 0x88888888u;
                px[0] = pal_lookup4s(s0, x0, P.x, P.y, P.z, P.w, one); px[1] = pal_lookup4s(__umulhi(s0, m16), __umulhi(x0, m16), P.x, P.y, P.z, P.w, one);
                px[2] = pal_lookup4s(s1, x1, P.x, P.y, P.z, P.w, one); px[3] = pal_lookup4s(__umulhi(s1, m16), __umulhi(x1, m16), P.x, P.y, P.z, P.w, one);
                px[4] = pal_lookup4s(s2, x2, P.x, P.y, P.z, P.w, one); px[5] = pal_lookup4s(__umulhi(s2, m16), __umulhi(x2, m16), P.x, P.y, P.z, P.w, one);
                px[6] = pal_lookup4s(s3, x3, P.x, P.y, P.z, P.w, one); px[7] = pal_lookup4s(__umulhi(s3, m16), __umulhi(x3, m16), P.x, P.y, P.z, P.w, one);
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) px[q] = bdw;
            }
            // ---- sprites of lines l0..l0+3 (CopySprites, patch:1615-1640: the first opaque pixel in OAM order wins,
            // and shows the background instead where it is behind an opaque background pixel). The lines' pixels go
            // to shared memory; lane group g evaluates the end of line l - 1 (the fetch line l draws) over the
            // visible sprites in OAM order, 8 candidates per round, and each lane holding one of the first 8 in range
            // writes that sprite's pixels as bytes (bit 7: taken by a sprite); within a round the pixels an earlier
            // sprite of the round covers are found from the other lanes' opaque masks, across rounds from bit 7.
            if (any) {
                u8* rowb = F.rows[g];
                uint4* rw = reinterpret_cast<uint4*>(rowb + 32u * j);
                rw[0] = make_uint4(px[0], px[1], px[2], px[3]);
                rw[1] = make_uint4(px[4], px[5], px[6], px[7]);
                __syncwarp();
                const int e = l - 1;
                const uint2 re = F.rec[e];
                const u32 ctrl = ((re.x >> 18) & 7u) << 3;
                const bool on = (re.y & 0x18u) && (re.y & (1u << 16));
                const u32 hgt = (ctrl & 0x20u) ? 16u : 8u;
                const u32* pages = F.chr[(re.y >> 12) & 3u];
                const u32 vofs = ((ctrl & 0x08u) && !(ctrl & 0x20u)) ? 0x1000u : 0u;
                const u32* spal = reinterpret_cast<const u32*>(&F.spal[(re.y >> 20) & 3u]);   // at the end of line e
                u32 nsp = 0;   // this lane group's sprites so far
                for (u32 c0 = 0; c0 < nv; c0 += 8) {   // warp-uniform trip count
                    const u32 c = c0 + j;
                    const u32 si = c < nv ? vis[c] : 0u;
                    const u32 wa = __shfl_sync(0xFFFFFFFFu, spA, si & 31u), wb = __shfl_sync(0xFFFFFFFFu, spB, si & 31u);
                    const u32 spw = si >= 32u ? wb : wa;
                    const u32 t = static_cast<u32>(e - static_cast<int>(spw & 0xFFu));
                    const bool in = on && c < nv && t < hgt;
                    const u32 gb = (__ballot_sync(0xFFFFFFFFu, in) >> (8u * g)) & 0xFFu;
                    const bool mine = in && nsp + __popc(gb & ((1u << j) - 1u)) < 8u;
                    const u32 attr = (spw >> 16) & 0xFFu, xx = spw >> 24;
                    // the sprite's row (every lane, no branches: the address stays inside the pattern tables):
                    // row tf of the sprite, vertical flip tf = h - 1 - t; rows 8-15 of an 8x16 sprite in its second tile
                    const u32 tile = (spw >> 8) & 0xFFu;
                    const u32 tf = (attr & 0x80u) ? hgt - 1u - t : t;
                    const u32 vadr = (hgt == 16u ? ((tile & 1u) << 12) + ((tile & 0xFEu) << 4) : (tile << 4) + vofs) + tf + (tf & 8u);
                    const u32 cwr = chr_sel(pages, vadr & 0x1FFFu);
                    const u32 cw = mine ? ((attr & 0x40u) ? nib_reverse(cwr) : cwr) : 0u;
                    const u32 om = nib_opaque8(cw);   // bit p: pixel p (screen x xx + p) is opaque; 0 unless mine
                    // pixels of this sprite that a sprite of the round before it covers: the lanes of the group below
                    // this one that hold a drawn sprite, one per trip (the trip count is the warp's largest number of
                    // such lanes, mostly 0 or 1)
                    const u32 info = (xx << 8) | om;
                    u32 cov = 0;
                    const u32 drawn = __ballot_sync(0xFFFFFFFFu, om != 0u);   // every lane (a full-warp vote)
                    u32 below = om ? (drawn >> (8u * g)) & ((1u << j) - 1u) : 0u;
                    const u32 kmax = __reduce_max_sync(0xFFFFFFFFu, __popc(below));
                    for (u32 k = 0; k < kmax; ++k) {
                        const u32 src = below ? static_cast<u32>(__ffs(below)) - 1u : j;
                        below &= below - 1u;
                        const u32 o = __shfl_sync(0xFFFFFFFFu, info, 8u * g + src);
                        const int d = static_cast<int>(o >> 8) - static_cast<int>(xx);   // other sprite's pixel q = my q + d
                        const u32 oq = src != j ? o & 0xFFu : 0u;
                        if (d > -8 && d < 8) cov |= d >= 0 ? oq << d : oq >> -d;
                    }
                    u32 wm = om & ~cov;
                    if (xx < 8u) wm &= 0xFFu << (8u - xx);   // screen x < 8 is cropped
                    if (wm) {
                        const u32 sw = spal[attr & 3u];
                        const u32 clo = __byte_perm(sw, 0u, cw) | 0x80808080u, chi = __byte_perm(sw, 0u, cw >> 16) | 0x80808080u;
                        // byte masks of the visible pixels 0-3 and 4-7
                        const u32 mlo = (((wm & 0xFu) * 0x00204081u) & 0x01010101u) * 0xFFu;
                        const u32 mhi = ((((wm >> 4) & 0xFu) * 0x00204081u) & 0x01010101u) * 0xFFu;
                        const u32 behm = (attr & 0x20u) ? 0xFFFFFFFFu : 0u;   // behind the background
                        // the 8 pixels (bytes x8 .. x8 + 7 of the row) as the 3 row words w0 .. w0 + 2 they touch
                        const int x8 = static_cast<int>(xx) - 8;
                        const int w0 = x8 >> 2;   // -2 .. 61; words before the row hold only cropped pixels (mask 0)
                        const u32 sh = 8u * (static_cast<u32>(x8) & 3u);
                        const u32 cwd[3] = {clo << sh, __funnelshift_l(clo, chi, sh), __funnelshift_l(chi, 0u, sh)};
                        const u32 mwd[3] = {mlo << sh, __funnelshift_l(mlo, mhi, sh), __funnelshift_l(mhi, 0u, sh)};
                        u32* roww = reinterpret_cast<u32*>(rowb);
#pragma unroll
                        for (int k = 0; k < 3; ++k) {
                            const int wi = w0 + k;
                            if (mwd[k] != 0u && wi >= 0) {
                                // bytes of this word no other lane of the round writes (claims are disjoint): read,
                                // then change only them, by an xor, while other lanes may change the rest
                                const u32 old = roww[wi];
                                const u32 taken = prmt_signed(old, 0u, 0xBA98u);         // bit 7: an earlier round's
                                const u32 bgop = prmt_signed(old << 1, 0u, 0xBA98u);     // bit 6: opaque background
                                const u32 m = mwd[k] & ~taken;
                                const u32 keep = m & bgop & behm;
                                const u32 val = (cwd[k] & ~keep) | ((old | 0x80808080u) & keep);
                                atomicXor(&roww[wi], (old ^ val) & m);
                            }
                        }
                    }
                    __syncwarp();
                    nsp += __popc(gb);
                }
                px[0] = rw[0].x; px[1] = rw[0].y; px[2] = rw[0].z; px[3] = rw[0].w;
                px[4] = rw[1].x; px[5] = rw[1].y; px[6] = rw[1].z; px[7] = rw[1].w;
            }
            if ((mask & 1u) && (mask & 0x18u)) {   // greyscale
#pragma unroll
                for (int q = 0; q < 8; ++q) px[q] &= 0x30303030u;
            }
            const int y = l - kObsY0;
            bool exact = false;
            if constexpr (kSplitLines) exact = ((F.split[l >> 5] >> (l & 31)) & 1u) != 0u;   // drawn by the walk
            if (exact) {
            } else if (!pack6) {
                uint4* row = reinterpret_cast<uint4*>(obs_out + static_cast<u64>(y) * kObsW + 32u * j);
                row[0] = make_uint4(px[0] & 0x3F3F3F3Fu, px[1] & 0x3F3F3F3Fu, px[2] & 0x3F3F3F3Fu, px[3] & 0x3F3F3F3Fu);
                if (j < 7) row[1] = make_uint4(px[4] & 0x3F3F3F3Fu, px[5] & 0x3F3F3F3Fu, px[6] & 0x3F3F3F3Fu, px[7] & 0x3F3F3F3Fu);
            } else {
                // 6-bit groups (bits 6-7 of each byte are dropped by the packing), joined into words by byte permutes
                u32 gq[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) gq[q] = pack_group6_loose(px[q], m30, m28);
                u32* row = reinterpret_cast<u32*>(obs_out + static_cast<u64>(y) * (kObsW / 4 * 3) + 24u * j);
                row[0] = __byte_perm(gq[0], gq[1], 0x4210);
                row[1] = __byte_perm(gq[1], gq[2], 0x5421);
                row[2] = __byte_perm(gq[2], gq[3], 0x6542);
                if (j < 7) {
                    row[3] = __byte_perm(gq[4], gq[5], 0x4210);
                    row[4] = __byte_perm(gq[5], gq[6], 0x5421);
                    row[5] = __byte_perm(gq[6], gq[7], 0x6542);
                }
            }
            __syncwarp();   // the staging rows are rewritten by the next iteration
        }
        for (int i = lane; i < kObsH / 4; i += 32) {   // emphasis bits of the 224 drawn lines
            u32 e4 = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) e4 |= ((F.rec[kObsY0 + 4 * i + k].y >> 5) & 7u) << (8 * k);
            reinterpret_cast<u32*>(emph_out)[i] = e4;
        }
    }

    __device__ void draw(u32 ge, u32 f, u8* obs_out, u8* emph_out, bool pack6) {
        const u64 sl = static_cast<u64>(ge) * 4 + f;
        const u32 bank = A.st.slot_bank[sl];
        h = A.st.log + (static_cast<u64>(ge) * kLogBanks + bank) * kLogBankWords;
        ev = h + kLogHdr;
        count = min(h[0] & ~kLogOverflow, kLogEv);
        kook = (h[15] & kLogKook) ? 1 : 0;
        chr_ram = slot_chr(ge, sl);
        {   // the frame's nametable into shared memory, its OAM into registers (2 entries per lane)
            const uint4* ntg = reinterpret_cast<const uint4*>(A.st.snap_nt + sl * kNtBytes);
            uint4* nts = reinterpret_cast<uint4*>(W.nt);
            const uint4 q0 = ntg[lane], q1 = ntg[lane + 32], q2 = ntg[lane + 64], q3 = ntg[lane + 96];
            const u32* oamw = reinterpret_cast<const u32*>(A.st.snap_oam + sl * kOamBytes);
            spA = oamw[lane];
            spB = oamw[lane + 32];
            __syncwarp();
            nts[lane] = q0; nts[lane + 32] = q1; nts[lane + 64] = q2; nts[lane + 96] = q3;
        }
        // header (patch:1318-1343)
        s.ctrl = h[1] & 0xFFu; s.mask = (h[1] >> 8) & 0xFFu; s.x = (h[1] >> 16) & 7u;
        s.v = h[2] & 0x7FFFu; s.t = (h[2] >> 16) & 0x7FFFu;
        if (lane < 8) {
            W.chr[lane] = (h[3 + (lane >> 2)] >> ((lane & 3) * 8)) & 0xFFu;
            W.pal[lane] = h[7 + lane];
        }
        __syncwarp();
        if (lane == 0) make_bgp();
        __syncwarp();
        s.mirroring = h[5] & 0xFFu;
        s.sh0 = s.sh1 = s.at = 0;
        s.blurp = 0; s.spork = 0; s.hit = 0; s.sphitx = 0x100u; s.sphitmask = 0; s.hit_x = 0;
        s.fb = 0; s.fsame = 0;
        s.spal[0] = s.spal[1] = s.spal[2] = s.spal[3] = 0;
        s.lazy = 0; s.lz_v = 0; s.lz_ctrl = 0; s.lz_mir = 0; s.lz_saved = 0;
        s.nf = 0; s.nd = 0;
        s.latch[0] = (h[5] >> 8) & 1u; s.latch[1] = (h[5] >> 16) & 1u;
        for (int i = 0; i < 4; ++i) s.creg[i] = (h[6] >> (8 * i)) & 0xFFu;
        s.cursor = 0;
        s.next_t = time_of(0);
        while (s.next_t < -16) next_event(false);
        if (s.mask & 0x18u) s.v = s.t;

        for (int l = 0; l < kObsY0 + kObsH; ++l) {
            const int start = l * 341 - 16;
            u32 w0, w1;   // this lane's 8 background pixels (colour | 0x40 transparent), byte k = pixel 8L+k
            if (s.next_t < start + 272) {
                exact_line(l);
                const uint2 q = reinterpret_cast<const uint2*>(W.px)[lane];
                w0 = q.x; w1 = q.y;
            } else {
                const uint4 P = W.bgp;   // byte 0 of each word: backdrop | 0x40
                const u32 bdw = (P.x & 0xFFu) * 0x01010101u;
                if (!(s.mask & 0x18u)) {
                    w0 = w1 = bdw;   // rendering off: backdrop, nothing fetched, v unchanged
                } else {
                    const u32 v0 = s.v;
                    u32 ca, c32 = 0;
                    if constexpr (BOARD == kMmc2) {
                        ca = mmc2_fast_fetch(v0, c32);
                    } else {
                        const LineFetch lf = line_fetch(v0);
                        ca = line_tile(lf, lane);
                        if (lane == 31 && s.sphitx != 0x100u && s.sphitx >= 241u) c32 = line_tile(lf, 32);
                    }
                    u32 cn = __shfl_down_sync(0xFFFFFFFFu, ca, 1);
                    // fetch 32 only feeds pixels 248..255 (right of the crop): needed for a sprite-0 check there
                    const bool need32 = s.sphitx != 0x100u && s.sphitx >= 241u;
                    if (need32 && lane == 31) cn = c32;
                    const u32 sel = __funnelshift_r(ca, cn, 4 * s.x);
                    if (s.mask & 0x08u) {
                        // colour 0 of every sub-palette shows the backdrop
                        w0 = pal_lookup4(sel, P.x, P.y, P.z, P.w);
                        w1 = pal_lookup4(sel >> 16, P.x, P.y, P.z, P.w);
                        if (lane == 0 && !(s.mask & 0x02u)) { w0 = bdw; w1 = bdw; }
                    } else {
                        w0 = w1 = bdw;
                    }
                    // sprite-0 check at the line end (p = 272): pixels sphitx..sphitx+7, x < 255
                    if (s.sphitx != 0x100u) {
                        const u32 t0 = ~w0 & 0x40404040u, t1 = ~w1 & 0x40404040u;   // opaque = colour, not 0x40
                        const u32 ob = ((t0 >> 6) & 1u) | ((t0 >> 13) & 2u) | ((t0 >> 20) & 4u) | ((t0 >> 27) & 8u) |
                                       (((t1 >> 6) & 1u) << 4) | (((t1 >> 13) & 2u) << 4) | (((t1 >> 20) & 4u) << 4) |
                                       (((t1 >> 27) & 8u) << 4);
                        const u32 sx = s.sphitx;
                        const u32 lo_l = sx >> 3;
                        const u32 olo = __shfl_sync(0xFFFFFFFFu, ob, lo_l & 31u);
                        const u32 ohi = __shfl_sync(0xFFFFFFFFu, ob, (lo_l + 1) & 31u);
                        const u32 win = ((olo | (lo_l + 1 < 32 ? (ohi << 8) : 0u)) >> (sx & 7u)) & 0xFFu;
                        const u32 lim = sx + 8u <= 255u ? 0xFFu : ((1u << (255u - sx)) - 1u);
                        const u32 hits = win & s.sphitmask & lim;
                        if (hits) { s.hit = 1; s.hit_x = sx + (__ffs(hits) - 1); s.sphitx = 0x100u; }
                    }
                    if constexpr (BOARD != kMmc2) {   // MMC2 keeps its shift registers (mmc2_fast_fetch)
                        s.lazy = 1; s.lz_v = v0; s.lz_ctrl = s.ctrl; s.lz_mir = s.mirroring; s.lz_saved = 0;
                    }
                    s.v = v_inc_y(v_inc_x_n(v0, 34));
                }
            }
            // CopySprites (patch:1615-1640) then greyscale
            if ((s.mask & 0x10u) && s.spork) {
                s.spork = 0;
                const RSprites& d = W.spr[s.fb ^ 1u];
                u32 snib = 0, sany = 0, sbeh = 0;
                const int base = static_cast<int>(lane) * 8;
                for (int i = static_cast<int>(s.nd) - 1; i >= 0; --i) {
                    const u32 meta = d.meta[i];
                    const int dx = static_cast<int>(meta >> 8) - base;
                    if (dx <= -8 || dx >= 8) continue;
                    const u32 cw = d.cw[i];
                    const u32 win = dx >= 0 ? (cw << (4 * dx)) : (cw >> (4 * -dx));
                    const u32 om = ((win | (win >> 1)) & 0x11111111u) * 0xFu;
                    const u32 pw = (meta & 3u) * 0x44444444u;
                    snib = (snib & ~om) | ((win | pw) & om);
                    sany |= om;
                    sbeh = (meta & 4u) ? (sbeh | om) : (sbeh & ~om);
                }
                if (lane == 0 && !(s.mask & 0x04u)) sany = 0;
                if (sany) {
                    const u32 c0 = pal_lookup4(snib, s.spal[0], s.spal[1], s.spal[2], s.spal[3]);
                    const u32 c1 = pal_lookup4(snib >> 16, s.spal[0], s.spal[1], s.spal[2], s.spal[3]);
                    const u32 any0 = nib_to_bytes(sany), any1 = nib_to_bytes(sany >> 16);
                    const u32 beh0 = nib_to_bytes(sbeh), beh1 = nib_to_bytes(sbeh >> 16);
                    const u32 tr0 = ((w0 & 0x40404040u) >> 6) * 0xFFu, tr1 = ((w1 & 0x40404040u) >> 6) * 0xFFu;
                    const u32 use0 = any0 & (~beh0 | tr0), use1 = any1 & (~beh1 | tr1);
                    w0 = (w0 & ~use0) | (c0 & use0);
                    w1 = (w1 & ~use1) | (c1 & use1);
                }
            }
            const u32 keep = ((s.mask & 1u) && (s.mask & 0x18u)) ? 0x30303030u : 0x3F3F3F3Fu;
            w0 &= keep;
            w1 &= keep;
            if (l >= kObsY0) {
                const int y = l - kObsY0;
                if (!pack6) {
                    if (lane >= 1 && lane <= 30)
                        reinterpret_cast<uint2*>(obs_out + static_cast<u64>(y) * kObsW)[lane - 1] = make_uint2(w0, w1);
                } else {
                    // 16 pixels of lanes L, L+1 (L odd) -> 12 bytes: four 24-bit groups of 4 colour numbers
                    const u32 g0 = pack_group6(w0), g1 = pack_group6(w1);
                    const u32 n0 = __shfl_down_sync(0xFFFFFFFFu, g0, 1), n1 = __shfl_down_sync(0xFFFFFFFFu, g1, 1);
                    if ((lane & 1u) && lane <= 29) {
                        u32* row = reinterpret_cast<u32*>(obs_out + static_cast<u64>(y) * (kObsW / 4 * 3)) + 3 * ((lane - 1) >> 1);
                        row[0] = g0 | (g1 << 24);
                        row[1] = (g1 >> 8) | (n0 << 16);
                        row[2] = (n0 >> 16) | (n1 << 8);
                    }
                }
                if (lane == 0) W.emph[y] = static_cast<u8>((s.mask >> 5) & 7u);
            }
            end_of_line(l);
        }
        __syncwarp();
        for (int i = lane; i < kObsH / 4; i += 32)
            reinterpret_cast<u32*>(emph_out)[i] = reinterpret_cast<const u32*>(W.emph)[i];
        __syncwarp();
    }
};

}  // namespace gr
