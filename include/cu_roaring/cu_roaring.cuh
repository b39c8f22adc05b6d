// cu_roaring B200 engine — umbrella header (drop-in for the reference
// include/cu_roaring/cu_roaring.cuh). Link with -lcuroaring_b200.
#pragma once
#include "cu_roaring/types.cuh"
#include "cu_roaring/detail/utils.cuh"
#include "cu_roaring/detail/promote.cuh"
#include "cu_roaring/detail/upload.cuh"
#include "cu_roaring/detail/upload_ids.cuh"
#include "cu_roaring/detail/decompress.cuh"
#include "cu_roaring/detail/set_ops.cuh"
#include "cu_roaring/detail/to_csr.cuh"
#include "cu_roaring/detail/filtered_topk.cuh"
#include "cu_roaring/device/roaring_view.cuh"
#include "cu_roaring/device/roaring_warp_query.cuh"
#include "cu_roaring/device/make_view.cuh"
#include "cu_roaring/filters/roaring_filter.cuh"
