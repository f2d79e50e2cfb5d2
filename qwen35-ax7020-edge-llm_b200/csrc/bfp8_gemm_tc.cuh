// bfp8_gemm_tc.cuh -- batched BFP8 GEMM on the tcgen05 tensor cores (sm_100a).
//
// Batched decode runs B sequences through the same weights, so each weight
// row meets B activation rows: a dense int8 contraction.  The int16 block-64
// activations (xq in [-16384, 16384], one f32 scale per 64-block) are stored
// as two signed int8 planes, xq = 256*hi + lo with lo the low byte of xq read
// as a signed int8 (-128..127) and hi = (xq - lo) / 256 (-64..64), so the
// tensor cores compute both halves of every block dot exactly in int32
// (tcgen05.mma kind::i8, one signed x signed MMA over both planes) and the
// epilogue recombines D = 256*Dhi + Dlo -- the same integer the batch-1
// kernel forms with dp2a.  Per block the epilogue adds
// float(D) * 2^(e-134) * xs to an f32 accumulator (order: blocks ascending,
// one fused multiply-add each), which agrees with the reference's NEON
// combine to a few ulp of the sum of |terms|.
//
// Activation layout ("planar int16"): planes [2][B][K] bytes (plane 0 = hi,
// plane 1 = lo) and block scales xs_t [K/64][ldxs] f32 (block-major, so one
// TMA box brings a stage's scales for a tile of batch columns).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "peer.cuh"

namespace qb {

// One GEMM of a (grouped) launch: y[B][M] = W[M][K] (BFP8) x X[B][K] (planar int16).
struct alignas(128) TcDesc {
    CUtensorMap tm_w;       // mantissas [M][K] u8, box 128 rows x 128 B, SWIZZLE_128B
    CUtensorMap tm_x;       // planes [2][B][K] u8, box 128 B x N rows x 2 planes, SWIZZLE_128B
    CUtensorMap tm_s;       // scales [nb][ldxs] f32, box N columns x 2 blocks
    const uint8_t* exps;    // [M][nb]
    float* y;               // [B][ldy]: row b of the output at y + b * ldy
    int32_t* dots;          // optional [B][M][nb]: exact block dots (verification)
    int M, K, B, nb;
    int unit_begin;         // first unit (row tile x column tile) of this GEMM; stream-K: first stage
    int n_nt;               // column tiles per row tile
    int ldy;                // output row stride (>= M)
    int tile_begin;         // stream-K launches: index of this GEMM's first tile among the launch's tiles
    const PeerOut* peer;    // optional (device memory): row-sharded GEMMs also store into every rank's output
};

// Column-tile width used for a batch of B rows (8, 16, 32, 64 or 128).
int tc_tile_n(int B);

// Fill `d` (host memory); false if a pointer, stride or size breaks the
// kernel's alignment rules.
bool tc_make_desc(TcDesc* d, float* y, const void* planes, const float* xs_t, int ldxs, const int8_t* mant,
                  const uint8_t* exps, int M, int K, int B, int32_t* dots, int ldy = 0);   // ldy 0: M

// Units (tiles: row tile x column tile) of one descriptor after tc_make_desc.
int tc_units(const TcDesc& d);

// Stream-K launches: every CTA takes an equal, contiguous share of the
// launch's K stages (tile after tile, each tile's stages in K order), so the
// work is balanced whatever the tile count.  A tile cut between CTAs is
// finished by the last of its pieces to complete, which adds the pieces'
// partial sums in K order.
constexpr int kTcTicketsPerTile = 16;   // one counter per epilogue warp of a tile
constexpr int kTcTileRowsPublic = 128;  // weight rows per tile (a partial slot holds B x 128 fp32)
int tc_stages(const TcDesc& d);          // K stages of one descriptor: tiles x ceil(nb / blocks per stage)
int tc_streamk_grid(int total_stages);   // CTAs of a stream-K launch
// Stream-K pays off when a launch has too few tiles to spread evenly over the
// SMs (whole-tile units, CTA c taking units c, c + G, ..., keep the tiles of
// neighbouring CTAs adjacent, which the L2 rewards when there are plenty).
bool tc_prefer_streamk(int tiles);
struct TcStreamK {
    float* partial;          // 2 x grid slots of B x 128 fp32 (pieces cut at CTA boundaries)
    unsigned int* tickets;   // kTcTicketsPerTile zeroed counters per tile of the launch (left zero)
    int total_stages;        // sum of tc_stages over the launch's descriptors (their unit_begin = first stage)
};

// GEMMs one launch takes (a grouped plan of more is split into launches).
constexpr int kTcMaxDescs = 160;

// Launch: `dev_descs` (device array of n descriptors with unit_begin set,
// largest K first) or, when it is null, the single descriptor `one`.  With
// `dots` the kernel also writes every exact block dot to desc.dots.
// `sync` (row-sharded plans): the last CTA publishes sig_epoch (its wait
// fields are unused: the quantizer that feeds the launch waits).
cudaError_t launch_gemm_tc(const TcDesc* dev_descs, const TcDesc* one, int n, int total_units, int B, bool dots,
                           unsigned int* err, cudaStream_t stream, const SyncArgs* sync = nullptr,
                           const TcStreamK* sk = nullptr);

// fp32 [B][K] -> planes [2][B][K] + xs_t [K/64][ldxs],
// the reference quantizer's arithmetic (bit-exact xq and scales).  With
// `sync`, every CTA first waits (bounded) for sync->wait_epoch from all ranks.
cudaError_t launch_quant_planes(const float* x, int B, int K, void* planes, float* xs_t, int ldxs,
                                cudaStream_t stream, const SyncArgs* sync = nullptr, unsigned int* err = nullptr);

}  // namespace qb
