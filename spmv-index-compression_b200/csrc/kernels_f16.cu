// kernels_f16.cu — kernel instantiations for __half values.
#define VALUE_TYPE __half
#define LAUNCH_TILES_NAME launch_tiles_f16
#define LAUNCH_VECTOR_NAME launch_vector_f16
#define TILES_OCCUPANCY_NAME tiles_occupancy_f16
#define LAUNCH_CLASSES_NAME launch_classes_f16
#define PREPARE_CLASSES_NAME prepare_classes_f16
#include "kernels_instantiate.cuh"
