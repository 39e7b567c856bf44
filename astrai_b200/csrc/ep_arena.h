// Layout descriptor of an expert-parallel symmetric arena (shared by the MoE
// kernels and their bindings). Offsets are bytes from each rank's arena base.
#pragma once

namespace astrai {

// Exchange phases; each has a row of arrival counters in every rank's flag block.
enum EPPhase : int { kPhDispatch = 0, kPhReturn = 1, kPhScatterBwd = 2, kPhReturnBwd = 3, kPhCounts = 4 };
constexpr int kEPPhases = 5;

struct EPArena {
  const long long* peer_base;  // [W] arena bases (this process's mappings)
  int rank, world;
  long long off_flags;   // [kEPPhases][W] u32 arrival counters, one row per phase, one column per source rank
  long long off_counts;  // [W][E] int32 routed-slot counts per expert, one row per source rank
  long long off_srcmap;  // [rows_cap] int64 (src_rank << 32 | slot)
  long long off_xin;     // [rows_cap, d] expert input block
  long long off_dyin;    // [rows_cap, d] expert output-gradient block
  long long off_ret;     // [slots_cap, d] returned expert outputs (forward)
  long long off_ret2;    // [slots_cap, d] returned input gradients (backward)
  long long off_xin8;    // [rows_cap, d] fp8 e4m3 expert input (fp8 dispatch; 0 when unused)
  long long off_xsc;     // [rows_cap, d / 128] fp32 block scales of off_xin8
  long long rows_cap, slots_cap;
  int d;
  unsigned* done;        // local grid-completion counter
  unsigned* expect;      // local [kEPPhases] rounds of each phase this rank has waited for
  int* err;
  unsigned long long wait_ns;
};

}  // namespace astrai
