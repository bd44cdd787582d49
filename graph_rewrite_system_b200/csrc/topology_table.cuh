// Layout of the per-xfer rewrite table (int32 rows of TAB_WIDTH), built by
// the host from the rule patterns (topology.py) and read by the topology and
// shard kernels.
#pragma once

namespace grs {

constexpr int TAB_MAXP = 4;          // ops per pattern
constexpr int TAB_MAXW = 4;          // qubit wires per pattern
constexpr int TAB_MAXE = 8;          // internal destination edges
constexpr int TAB_SRC_LEN = 0, TAB_DST_LEN = 1, TAB_DST_TYPES = 2, TAB_NWIRES = 6,
              TAB_WIRES = 7, TAB_NINT = 7 + TAB_MAXW * 8, TAB_INT = TAB_NINT + 1,
              TAB_WIDTH = TAB_INT + TAB_MAXE * 4;

}  // namespace grs
