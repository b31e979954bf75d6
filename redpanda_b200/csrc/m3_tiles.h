// The compiled lane tilings.  R/T = rotational/tracking lanes per thread per
// channel (state lanes are split over 4 threads); NDF / NDB = channels per
// thread in the forward/step and in the backward kernel; NTHB = backward CTA
// size (128 = one warpgroup; 256 = two, each with its own half of Tensor
// Memory).  A backward CTA that needs 256 or fewer TMEM columns shares its SM
// with a second one, so the two CTAs' barriers and flushes overlap each
// other's arithmetic.
// NDB = 0: forward and step only (the backward needs R + T <= 16).
// GS = 1: the backward keeps each step's rotational gates exp*cos and exp*sin
// in Tensor Memory next to the state (so its reverse pass evaluates no
// transcendental), which halves its chunk to 8 steps; the forward then writes
// its checkpoints every 8 steps instead of 16.  Needs NDB*(R+T+2R) <= 32.
// Any (n_rot, n_track) split is served by the smallest tiling with
// R >= ceil(n_rot/4) and T >= ceil(n_track/4); surplus lanes are virtual.
#pragma once

// X(R, T, NDF, NDB, NTHB, GS)
#define M3_TILE_LIST(X) \
  X(3, 1, 8, 4, 256, 0)    /* N=16, 12 rot + 4 track (config 0)               */ \
  X(4, 4, 4, 2, 128, 1)    /* N=32, 16 rot + 16 track (configs 1, 2, 4)       */ \
  X(6, 2, 4, 2, 256, 0)    /* N=32, 24 rot + 8 track (config 3, Search Mamba) */ \
  X(2, 1, 8, 4, 256, 0)    /* N=12, 8 rot + 4 track; N=8, 6 rot + 2 track     */ \
  X(4, 0, 8, 4, 256, 0)    /* N=16, no tracking                               */ \
  X(2, 0, 8, 4, 256, 0)    /* N=8, no tracking                                */ \
  X(8, 0, 4, 2, 256, 0)    /* N=32, no tracking                               */ \
  X(12, 4, 2, 2, 128, 0)   /* N=64, 48 rot + 16 track                         */ \
  X(16, 0, 2, 2, 128, 0)   /* N=64, no tracking                               */ \
  X(8, 8, 2, 2, 128, 0)    /* fallback: up to 32 rot + 32 track               */ \
  X(16, 16, 1, 0, 128, 0)  /* fallback: up to 64 rot + 64 track               */

// Small-batch tilings: the same lane splits with 2 channels per thread in the
// forward (64-channel tiles) and 128-thread backward CTAs, used when the
// regular tiling would give the scan fewer CTAs than the GPU has SMs (config 0
// at B=8; a search priming one board).  A cell's arithmetic and the y / dΔ /
// du reductions depend only on the lane split (R, T), so y, the checkpoints,
// the final state, dΔ and du are the same bits under both tilings; dB/dC
// (summed over channel tiles) and dA (over batch groups) follow the tiling's
// partition and agree within rounding.  Same X(R, T, NDF, NDB, NTHB, GS)
// fields as M3_TILE_LIST.
#define M3_SMALL_TILE_LIST(X) \
  X(3, 1, 2, 2, 128, 0)    /* N=16, 12 rot + 4 track (config 0)               */ \
  X(4, 4, 2, 2, 128, 1)    /* N=32, 16 rot + 16 track                         */ \
  X(6, 2, 2, 2, 128, 0)    /* N=32, 24 rot + 8 track (config 3)               */
