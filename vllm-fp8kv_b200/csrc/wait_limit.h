// wait_limit.h -- iteration limit of the decode kernels' bounded on-chip waits.
#pragma once
#include <stdint.h>

namespace fp8mla {
// try_wait suspends for a hardware-chosen interval per call (about 87 ns on
// B200, so 2^22 calls take about 0.4 s): well beyond the longest legitimate
// wait of a CTA (its whole MMA chain, tens of microseconds), yet a broken
// protocol ends in under a second with the timeout recorded.
constexpr uint32_t kMaxWaitIters = 1u << 22;
}  // namespace fp8mla
