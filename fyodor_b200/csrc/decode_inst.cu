// decode_inst.cu - one instantiation of the persistent decode kernel. The
// build compiles this file once per variant with -DFYB_DK_HD=<head dimension>
// -DFYB_DK_G=<query heads per KV head>; decode.cu reaches each one through
// decode_entry_<HD>_<G>(). Compiled without the two macros it defines nothing.
#if defined(FYB_DK_HD) && defined(FYB_DK_G)
#include "decode_kernel.cuh"

#define FYB_DK_NAME3(HD, G) decode_entry_##HD##_##G
#define FYB_DK_NAME(HD, G) FYB_DK_NAME3(HD, G)

namespace fyb {

DecodeKernel FYB_DK_NAME(FYB_DK_HD, FYB_DK_G)()
{
    return decode_kernel<FYB_DK_HD, FYB_DK_G>;
}

}  // namespace fyb
#endif
