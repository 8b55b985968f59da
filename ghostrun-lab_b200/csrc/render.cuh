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

struct RSprites {   // per warp, shared memory: a sprite line (FetchSpriteData / RefreshSprites)
    u32 cw[8];      // colour nibbles of the 8 pixels left to right (flip applied), 0 = transparent
    u32 meta[8];    // palette attr (bits 0-1) | behind (bit 2) | x << 8
    u32 opq0;       // first fetched sprite: bit k = its pixel k (screen order) is opaque (sprite-0 hit data)
    u32 n;
};

struct RWarp {      // per-warp shared scratch
    RSprites spr[2];     // fetched / drawn (double buffer)
    u32 pal[8];          // palette RAM of the replay (4 bytes per word)
    u32 chr[8];          // 1 KB CHR page per slot (paged boards)
    u32 lzchr[8];        // CHR pages of the line whose shift registers are kept lazily
    alignas(16) u8 nt[2048];  // the frame's nametable snapshot
    alignas(16) u8 px[256];   // exact-path line buffer
    u8 emph[224];
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
    u32 e0, count;       // global env range of this launch (game slice)
    u32 frames;          // frames per env to draw (4)
    u32 chrx_smem;       // 1: the cart's pattern table is staged in shared memory (8 KB CHR ROM boards)
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

// nibble mask (4 nibbles, each 0 or 0xF, low 16 bits) -> byte mask
__device__ __forceinline__ u32 nib_to_bytes(u32 nm16) { return __byte_perm(0u, 0xFFFFFFFFu, nm16 & 0x4444u); }

// 4 colour numbers (bytes) -> one 24-bit 6-bit group (rl/csrc/rlenv.cu:126-134 layout)
__device__ __forceinline__ u32 pack_group6(u32 w) {
    return (w & 0x3Fu) | ((w >> 2) & 0xFC0u) | ((w >> 4) & 0x3F000u) | ((w >> 6) & 0xFC0000u);
}

struct RState {
    u32 v, t, x, ctrl, mask, mirroring;
    u32 sh0, sh1, at;    // tile shift registers (low 16 bits) and attribute latch
    u32 blurp, spork, hit, sphitx, sphitmask, hit_x;
    u32 fb;              // which of the two sprite buffers is `fetched`
    u32 spal[4];         // sprite palette taken at RefreshSprites (& 0x3F)
    u32 lazy, lz_v, lz_ctrl, lz_mir;   // shift registers not yet materialised: fetches 32 / 33 of the line at lz_v
    u32 cursor;
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

    __device__ Renderer(const RenderArgs& a, u32 ln, const u32* cx, const u32* sp, RWarp& w)
        : A(a), lane(ln), chrx(cx), spread(sp), W(w) {}

    __device__ __forceinline__ int ev_time(u32 i) const { return fceumm_time(ev[2 * i] & 0x1FFFFu, kook); }
    __device__ __forceinline__ u32 pal_byte(u32 i) const { return reinterpret_cast<const u8*>(W.pal)[i]; }
    __device__ __forceinline__ static constexpr bool paged() { return BOARD == kMmc1 || BOARD == kMmc3; }

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
                if (lane == 0) reinterpret_cast<u8*>(W.pal)[aux & 31u] = static_cast<u8>(value);
                __syncwarp();
                s.v = (s.v + inc) & 0x7FFFu;
                break;
            case kEvChr:
                __syncwarp();
                if (lane == 0) W.chr[aux & 7u] = value;
                __syncwarp();
                break;
            case kEvMirror: s.mirroring = value; break;
            default: break;
        }
    }

    // The shift registers after the last fast line: its fetches 32 and 33.
    __device__ void materialize_shift() {
        if (!s.lazy) return;
        __syncwarp();
        const u32 c32 = fetch(v_inc_x_n(s.lz_v, 32), s.lz_ctrl, s.lz_mir, W.lzchr);
        const u32 c33 = fetch(v_inc_x_n(s.lz_v, 33), s.lz_ctrl, s.lz_mir, W.lzchr);
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
                const u32 p0 = chr_byte(W.chr, vadr), p1 = chr_byte(W.chr, vadr + 8u);
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
        while (s.cursor < count && ev_time(s.cursor) < start + 272) {
            const u32 kind = ev[2 * s.cursor] >> 24;
            if (kind != kEvDataWrite && kind != kEvPalette)
                update(ev_time(s.cursor) + 3 * static_cast<int>((ev[2 * s.cursor] >> 17) & 0xFu) - start);
            apply(s.cursor++, true);
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
            RSprites& f = W.spr[s.fb];
            const u32 c = s.ctrl;
            const u32 hgt = (c & 0x20u) ? 16u : 8u;
            const bool in0 = static_cast<u32>(l - static_cast<int>(spA & 0xFFu)) < hgt;
            const bool in1 = static_cast<u32>(l - static_cast<int>(spB & 0xFFu)) < hgt;
            const u32 b0 = __ballot_sync(0xFFFFFFFFu, in0), b1 = __ballot_sync(0xFFFFFFFFu, in1);
            s.blurp = b0 & 1u;
            u32 n = 0;
            if (b0 | b1) {
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
            }
            if (lane == 0) f.n = n;
            __syncwarp();
        }
        while (s.cursor < count && ev_time(s.cursor) < start + 278) apply(s.cursor++, true);
        if (s.mask & 0x18u) s.v = (s.v & 0xFBE0u) | (s.t & 0x041Fu);
        while (s.cursor < count && ev_time(s.cursor) < start + 341) apply(s.cursor++, true);
        if (s.mask & 0x10u) {
            s.spork = 0;
            const RSprites& f = W.spr[s.fb];
            if (f.n != 0) {
                s.fb ^= 1u;    // drawn = fetched (the other buffer becomes the next fetch target)
                for (int q = 0; q < 4; ++q) s.spal[q] = W.pal[4 + q] & 0x3F3F3F3Fu;
                if (s.blurp && !s.hit && f.opq0) {
                    s.sphitx = f.meta[0] >> 8;
                    s.sphitmask = f.opq0;
                }
                s.spork = 1;
            }
        }
    }

    __device__ void draw(u32 ge, u32 f, u8* obs_out, u8* emph_out, bool pack6) {
        const u64 sl = static_cast<u64>(ge) * 4 + f;
        const u32 bank = A.st.slot_bank[sl];
        h = A.st.log + (static_cast<u64>(ge) * kLogBanks + bank) * kLogBankWords;
        ev = h + kLogHdr;
        count = min(h[0] & ~kLogOverflow, kLogEv);
        kook = (h[15] & kLogKook) ? 1 : 0;
        chr_ram = (A.cart.chr == nullptr && A.st.snap_chr) ? A.st.snap_chr + sl * kChrRamBytes : nullptr;
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
        if (lane == 0) { W.spr[0].n = 0; W.spr[1].n = 0; }
        __syncwarp();
        s.mirroring = h[5] & 0xFFu;
        s.sh0 = s.sh1 = s.at = 0;
        s.blurp = 0; s.spork = 0; s.hit = 0; s.sphitx = 0x100u; s.sphitmask = 0; s.hit_x = 0;
        s.fb = 0;
        s.spal[0] = s.spal[1] = s.spal[2] = s.spal[3] = 0;
        s.lazy = 0; s.lz_v = 0; s.lz_ctrl = 0; s.lz_mir = 0;
        s.cursor = 0;
        while (s.cursor < count && ev_time(s.cursor) < -16) apply(s.cursor++, false);
        if (s.mask & 0x18u) s.v = s.t;

        for (int l = 0; l < kObsY0 + kObsH; ++l) {
            const int start = l * 341 - 16;
            u32 w0, w1;   // this lane's 8 background pixels (colour | 0x40 transparent), byte k = pixel 8L+k
            if (s.cursor < count && ev_time(s.cursor) < start + 272) {
                exact_line(l);
                const uint2 q = reinterpret_cast<const uint2*>(W.px)[lane];
                w0 = q.x; w1 = q.y;
            } else {
                const u32 bd = (pal_byte(0) & 0x3Fu) | 0x40u;
                const u32 bdw = bd * 0x01010101u;
                if (!(s.mask & 0x18u)) {
                    w0 = w1 = bdw;   // rendering off: backdrop, nothing fetched, v unchanged
                } else {
                    const u32 v0 = s.v;
                    const u32 ca = fetch(v_inc_x_n(v0, lane), s.ctrl, s.mirroring, W.chr);
                    u32 cn = __shfl_down_sync(0xFFFFFFFFu, ca, 1);
                    // fetch 32 only feeds pixels 248..255 (right of the crop): needed for a sprite-0 check there
                    const bool need32 = s.sphitx != 0x100u && s.sphitx >= 241u;
                    if (need32 && lane == 31) cn = fetch(v_inc_x_n(v0, 32), s.ctrl, s.mirroring, W.chr);
                    const u32 sel = __funnelshift_r(ca, cn, 4 * s.x);
                    if (s.mask & 0x08u) {
                        // colour 0 of every sub-palette shows the backdrop
                        const u32 P0 = (W.pal[0] & 0x3F3F3F00u) | bd, P1 = (W.pal[1] & 0x3F3F3F00u) | bd;
                        const u32 P2 = (W.pal[2] & 0x3F3F3F00u) | bd, P3 = (W.pal[3] & 0x3F3F3F00u) | bd;
                        w0 = pal_lookup4(sel, P0, P1, P2, P3);
                        w1 = pal_lookup4(sel >> 16, P0, P1, P2, P3);
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
                    s.lazy = 1; s.lz_v = v0; s.lz_ctrl = s.ctrl; s.lz_mir = s.mirroring;
                    if constexpr (paged()) { if (lane < 8) W.lzchr[lane] = W.chr[lane]; }
                    s.v = v_inc_y(v_inc_x_n(v0, 34));
                }
            }
            // CopySprites (patch:1615-1640) then greyscale
            if ((s.mask & 0x10u) && s.spork) {
                s.spork = 0;
                const RSprites& d = W.spr[s.fb ^ 1u];
                u32 snib = 0, sany = 0, sbeh = 0;
                const int base = static_cast<int>(lane) * 8;
                for (int i = static_cast<int>(d.n) - 1; i >= 0; --i) {
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
