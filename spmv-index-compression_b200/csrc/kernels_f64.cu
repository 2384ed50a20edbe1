// kernels_f64.cu — kernel instantiations for double values.
#define VALUE_TYPE double
#define LAUNCH_TILES_NAME launch_tiles_f64
#define LAUNCH_VECTOR_NAME launch_vector_f64
#define TILES_OCCUPANCY_NAME tiles_occupancy_f64
#define LAUNCH_CLASSES_NAME launch_classes_f64
#define PREPARE_CLASSES_NAME prepare_classes_f64
#include "kernels_instantiate.cuh"
