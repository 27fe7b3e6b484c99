// Layout check of the C ABI: the sizes of the structs a caller fills, so a binding built against another version
// of include/psgd_b200.h is refused before any launch reads a misaligned item array.
#include "psgd_b200.h"

extern "C" int psgd_struct_sizes(long long* sizes, int n) {
  const long long all[] = {
      (long long)sizeof(PsgdGemmSpec),   (long long)sizeof(PsgdPrepItem),      (long long)sizeof(PsgdNlbPrepItem),
      (long long)sizeof(PsgdFactorItem), (long long)sizeof(PsgdSkewItem),      (long long)sizeof(PsgdRotItem),
      (long long)sizeof(PsgdTraceItem),  (long long)sizeof(PsgdApplyItem),     (long long)sizeof(PsgdBalanceFactor),
      (long long)sizeof(PsgdBalanceParam), (long long)sizeof(PsgdSymItem),    (long long)sizeof(PsgdNlbFinishItem),
      (long long)sizeof(PsgdPermuteItem)};
  const int count = (int)(sizeof(all) / sizeof(all[0]));
  if (sizes == nullptr) return count;
  for (int i = 0; i < n && i < count; ++i) sizes[i] = all[i];
  return count;
}
