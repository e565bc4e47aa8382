// decode_inst.cu - one instantiation of the persistent decode kernel. The
// build compiles this file once per variant with -DFYB_DK_DF=<0 barrier form,
// 1 dataflow form> -DFYB_DK_HD=<head dimension> -DFYB_DK_G=<query heads per KV
// head>; decode.cu reaches each one through decode_entry_<DF>_<HD>_<G>().
// Compiled without the three macros it defines nothing.
#if defined(FYB_DK_DF) && defined(FYB_DK_HD) && defined(FYB_DK_G)
#include "decode_kernel.cuh"
#include "decode_df.cuh"

#define FYB_DK_NAME3(DF, HD, G) decode_entry_##DF##_##HD##_##G
#define FYB_DK_NAME(DF, HD, G) FYB_DK_NAME3(DF, HD, G)

namespace fyb {

DecodeKernel FYB_DK_NAME(FYB_DK_DF, FYB_DK_HD, FYB_DK_G)()
{
#if FYB_DK_DF
    return decode_df_kernel<FYB_DK_HD, FYB_DK_G>;
#else
    return decode_kernel<FYB_DK_HD, FYB_DK_G>;
#endif
}

}  // namespace fyb
#endif
