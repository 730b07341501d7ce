// prefill.hpp -- tile geometry shared by the prefill kernels (prefill.cu) and the host code.
#pragma once
#include <cstdint>

#include "internal.hpp"

namespace ugb {

constexpr int kPrefillTile = 128;                     // rows (tokens or weight rows) per tile
constexpr int kPrefillTileBytes = kPrefillTile * 32;  // one tile x one 32-wide K-block of int8

ugb_status init_prefill_kernels(ugb_ctx *ctx);

}  // namespace ugb
