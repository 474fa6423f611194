// Link-time stand-ins -- TEST INFRASTRUCTURE ONLY.
//
// src/core/position.cpp references three subsystems that the NN oracle never
// exercises: Syzygy probing (position.cpp's tablebase helpers), the search
// transposition table (prefetch in do_move when a TT pointer is passed; the
// harness always passes nullptr) and UCI square formatting (FEN/debug output).
// Linking their real sources would drag in the whole search and UCI stack, so
// these definitions satisfy the linker and fail loudly if ever reached.
#include "core/position.h"
#include "search/tt.h"
#include "syzygy/tbprobe.h"
#include "uci/uci.h"

#include <cstdio>
#include <cstdlib>

namespace MetalFish {
namespace Tablebases {
int MaxCardinality = 0;
WDLScore probe_wdl(Position &, ProbeState *) {
  std::fprintf(stderr, "oracle stub: Tablebases::probe_wdl reached\n");
  std::abort();
}
int probe_dtz(Position &, ProbeState *) {
  std::fprintf(stderr, "oracle stub: Tablebases::probe_dtz reached\n");
  std::abort();
}
} // namespace Tablebases
TTEntry *TranspositionTable::first_entry(const Key) const {
  std::fprintf(stderr, "oracle stub: TranspositionTable::first_entry reached\n");
  std::abort();
}
std::string UCIEngine::square(Square s) {
  std::string r;
  r += char('a' + int(s) % 8);
  r += char('1' + int(s) / 8);
  return r;
}
} // namespace MetalFish
