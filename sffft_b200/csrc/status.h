// Status codes shared by the kernels, the C ABI and the CLI.
#pragma once

#define SFFFT_OK 0
#define SFFFT_ERR_INVALID_ARGUMENT 1   // bad size, null pointer, unknown enum value
#define SFFFT_ERR_UNSUPPORTED 2        // length / plan / dtype combination not in the catalog
#define SFFFT_ERR_CUDA 3               // a CUDA runtime call failed (see sffft_last_cuda_error)
#define SFFFT_ERR_DEVICE 4             // device is not sm_100 / lacks shared memory for the plan
#define SFFFT_ERR_TIMEOUT 5            // a device-side barrier wait exceeded its limit
#define SFFFT_ERR_NO_MATCH 6           // selector found no candidate within the error budget
#define SFFFT_ERR_ALLOC 7              // device allocation failed
#define SFFFT_ERR_SCRATCH_LIMIT 8      // problem too large for the allocation-free entry point's scratch
