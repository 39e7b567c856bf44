// Layout descriptor of an expert-parallel symmetric arena (shared by the MoE
// kernels and their bindings). Offsets are bytes from each rank's arena base.
#pragma once

namespace astrai {

struct EPArena {
  const long long* peer_base;  // [W] arena bases (this process's mappings)
  int rank, world;
  long long off_flags;   // [4][W] u32 epochs, one row per phase
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
  int* err;
  unsigned long long wait_ns;
};

}  // namespace astrai
