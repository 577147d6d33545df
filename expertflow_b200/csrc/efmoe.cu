// efmoe.cu -- single translation unit of libefmoe.so (the device error word and
// the kernels are shared without relocatable device code).
#include "ef_permute.cu"
#include "ef_router.cu"
#include "ef_dequant.cu"
#include "ef_qmv.cu"
#include "ef_qgemm.cu"
#include "ef_qgemm2.cu"
#include "ef_api.cu"
#include "ef_store.cu"
#include "ef_kquant.cu"
#include "ef_pool.cu"
#include "ef_ep.cu"
#include "ef_noalloc.cu"
