"""ctypes binding of libfbgpu.so (include/fbgpu.h, include/fb_engine.h).

The library is built in-tree (ferrisboost_b200/build.py).  Importing this
module without the library, or calling a device entry point without a CUDA
device, raises: there is no CPU fallback behind the GPU API.
"""
import ctypes as C
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libfbgpu.so"

P = C.c_void_p
f32p = C.POINTER(C.c_float)
f64p = C.POINTER(C.c_double)
i64p = C.POINTER(C.c_int64)
u64p = C.POINTER(C.c_uint64)
u32p = C.POINTER(C.c_uint32)
i32p = C.POINTER(C.c_int32)
u16p = C.POINTER(C.c_uint16)
u8p = C.POINTER(C.c_uint8)
i8p = C.POINTER(C.c_int8)


class FbParams(C.Structure):
    _fields_ = [
        ("objective", C.c_int32), ("grow_policy", C.c_int32), ("max_depth", C.c_uint32),
        ("max_leaves", C.c_uint32), ("max_bin", C.c_uint32), ("eta", C.c_float), ("reg_lambda", C.c_float),
        ("gamma", C.c_float), ("min_child_weight", C.c_float), ("alpha", C.c_float),
        ("max_delta_step", C.c_float), ("scale_pos_weight", C.c_float), ("subsample", C.c_float),
        ("colsample_bytree", C.c_float), ("base_score", C.c_float), ("seed", C.c_uint64),
        ("max_cat_to_onehot", C.c_uint32), ("max_cat_threshold", C.c_uint32), ("nthread", C.c_int32),
        ("gpu_math", C.c_int32), ("device", C.c_int32), ("monotone", i8p), ("num_class", C.c_uint32),
        ("class_margins", f32p),
    ]


class FbgpuConfig(C.Structure):
    _fields_ = [
        ("device", C.c_int32), ("n_features", C.c_uint32), ("n_rows", C.c_uint64), ("n_rows_global", C.c_uint64),
        ("row_offset", C.c_uint64), ("max_depth", C.c_uint32), ("max_leaves", C.c_uint32),
        ("hist_smem_bytes", C.c_uint32), ("gpu_math", C.c_int32),
    ]


class FbgpuTreeParams(C.Structure):
    _fields_ = [
        ("eta", C.c_float), ("reg_lambda", C.c_float), ("gamma", C.c_float), ("min_child_weight", C.c_float),
        ("alpha", C.c_float), ("max_delta_step", C.c_float), ("max_depth", C.c_uint32),
        ("max_leaves", C.c_uint32), ("max_cat_to_onehot", C.c_uint32), ("max_cat_threshold", C.c_uint32),
        ("grow_policy", C.c_int32), ("monotone", i8p),
    ]


class FbgpuTreeOut(C.Structure):
    _fields_ = [
        ("capacity", C.c_uint32), ("n_nodes", C.c_uint32), ("left", i32p), ("right", i32p), ("feat", u32p),
        ("bin", u32p), ("gain", f32p), ("leaf", f32p), ("hess", f32p), ("flags", u32p), ("cats", u32p),
        ("cat_words", C.c_uint32), ("reserved", C.c_uint32),
    ]


class FbgpuSplit(C.Structure):
    _fields_ = [
        ("found", C.c_uint32), ("feat", C.c_uint32), ("bin", C.c_uint32), ("missing_left", C.c_uint32),
        ("gain", C.c_float), ("categorical", C.c_uint32), ("left_grad", C.c_int64), ("left_hess", C.c_int64),
        ("right_grad", C.c_int64), ("right_hess", C.c_int64), ("cats", C.c_uint32 * 8),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    # include/fbgpu.h
    "fbgpu_last_error": (C.c_char_p, [P]),
    "fbgpu_device_count": (C.c_int32, []),
    "fbgpu_launch_count": (C.c_uint64, []),
    "fbgpu_ctx_create": (C.c_int, [C.POINTER(FbgpuConfig), C.POINTER(P)]),
    "fbgpu_ctx_destroy": (None, [P]),
    "fbgpu_set_features": (C.c_int, [P, u32p, u8p, u8p]),
    "fbgpu_upload_block": (C.c_int, [P, u32p, C.c_uint32, C.c_uint32, P]),
    "fbgpu_set_labels": (C.c_int, [P, f32p, f32p, f32p, C.c_float]),
    "fbgpu_upload_and_quantize_gpair": (C.c_int, [P, f32p, C.c_uint64, C.c_uint64, C.c_uint64, f64p, i64p]),
    "fbgpu_upload_gpair": (C.c_int, [P, i64p, f64p, i64p]),
    "fbgpu_round_from_exp": (C.c_int, [P, C.c_int32, f32p, C.c_uint64, C.c_uint64, C.c_uint64, f64p]),
    "fbgpu_round_device": (C.c_int, [P, C.c_int32, C.c_int32, C.c_uint64, C.c_uint64, C.c_uint64, f64p, i64p]),
    "fbgpu_set_outputs": (C.c_int, [P, C.c_uint32, f32p]),
    "fbgpu_multiclass_gradients": (C.c_int, [P, C.c_int32]),
    "fbgpu_quantize_class": (C.c_int, [P, C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint64, C.c_int32, f64p, i64p]),
    "fbgpu_set_output_column": (C.c_int, [P, C.c_uint32]),
    "fbgpu_build_tree": (C.c_int, [P, C.POINTER(FbgpuTreeParams), u8p, C.POINTER(FbgpuTreeOut)]),
    "fbgpu_download_margins": (C.c_int, [P, f32p]),
    "fbgpu_nccl_unique_id": (C.c_int, [u8p]),
    "fbgpu_ctx_set_comm": (C.c_int, [P, u8p, C.c_int32, C.c_int32, C.c_uint32]),
    "fbgpu_exact_exp_available": (C.c_int32, [C.POINTER(C.c_char_p)]),
    "fbgpu_expf_check": (C.c_int, [C.c_int32, C.c_uint32, C.c_uint32, u64p, u32p]),
    "fbgpu_histogram": (C.c_int, [P, u32p, C.c_uint64, i64p, i64p]),
    "fbgpu_eval_split": (C.c_int, [P, i64p, i64p, f64p, C.POINTER(FbgpuTreeParams), C.c_float, C.c_float, u8p,
                                   C.POINTER(FbgpuSplit)]),
    "fbgpu_partition": (C.c_int, [P, u32p, C.c_uint64, C.c_uint32, C.c_uint32, C.c_int32, u32p, u32p, u64p]),
    "fbgpu_partition_set": (C.c_int, [P, u32p, C.c_uint64, C.c_uint32, C.c_int32, u32p, C.c_uint32, u32p, u64p]),
    "fbgpu_ctx_cat_words": (C.c_uint32, [P]),
    "fbgpu_split_cats": (C.c_int, [P, u32p, C.c_uint32]),
    "fbgpu_partition_noalloc": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, P, C.c_uint64,
                                         C.c_uint32, C.c_int32, u32p, P, P, P]),
    "fbgpu_hist_atomic_ceiling": (C.c_int, [C.c_int32, C.c_int32, C.c_uint32, f64p]),
    "fbgpu_model_create": (C.c_int, [C.c_int32, C.c_uint32, C.c_uint32, u32p, i32p, i32p, u32p, f32p, u8p, f32p,
                                     u32p, u32p, u32p, C.c_uint64, C.c_float, C.POINTER(P)]),
    "fbgpu_model_destroy": (None, [P]),
    "fbgpu_predict": (C.c_int, [P, f32p, C.c_uint64, f32p]),
    "fbgpu_predict_device": (C.c_int, [P, P, C.c_uint64, P, P]),
    "fbgpu_shap": (C.c_int, [P, f32p, C.c_uint64, f32p]),
    "fbgpu_shap_device": (C.c_int, [P, P, C.c_uint64, P, P]),
    "fbgpu_explain": (C.c_int, [P, C.c_int32, f32p, C.c_uint64, f32p]),
    "fbgpu_explain_device": (C.c_int, [P, C.c_int32, P, C.c_uint64, P, P]),
    # include/fb_engine.h
    "fb_default_params": (None, [C.POINTER(FbParams)]),
    "fb_last_error": (C.c_char_p, []),
    "fb_dataset_from_dense": (P, [f32p, C.c_uint64, C.c_uint32, C.c_uint32, f32p, u8p, C.c_int32]),
    "fb_dataset_with_cuts": (P, [f32p, C.c_uint64, C.c_uint32, f32p, u32p, u8p, C.c_int32]),
    "fb_dataset_on_device": (P, [f32p, C.c_uint64, C.c_uint32, C.c_uint32, f32p, u8p, f32p, u32p, C.c_int32,
                                 C.c_int32]),
    "fb_dataset_on_device_columns": (P, [f32p, C.c_uint64, C.c_uint32, C.c_uint32, f32p, u8p, f32p, u32p,
                                         C.c_int32, C.c_int32]),
    "fb_dataset_device": (C.c_int32, [P]),
    "fb_sketch_features": (C.c_int64, [f32p, C.c_uint64, C.c_uint32, C.c_uint32, f32p, u8p, u32p, C.c_uint32,
                                       C.c_int32, f32p, u32p, C.c_uint64]),
    "fb_sketch_features_device": (C.c_int64, [f32p, C.c_uint64, C.c_uint32, C.c_uint32, f32p, u8p, u32p, C.c_uint32,
                                              C.c_int32, C.c_int32, f32p, u32p, C.c_uint64]),
    "fb_label_mean": (C.c_float, [f32p, f32p, C.c_uint64]),
    "fb_label_mean_f64": (C.c_double, [f32p, C.c_uint64]),
    "fb_initial_base_score": (C.c_float, [C.c_int32, f32p, f32p, C.c_uint64, C.c_float]),
    "fb_class_margins": (C.c_int32, [f32p, f32p, C.c_uint64, C.c_uint32, f32p]),
    "fb_dataset_free": (None, [P]),
    "fb_dataset_rows": (C.c_uint64, [P]),
    "fb_dataset_cuts": (C.c_int64, [P, f32p, u32p, C.c_uint64]),
    "fb_dataset_column": (C.c_int32, [P, C.c_uint32, u16p]),
    "fb_booster_create": (P, [P, f32p, f32p, C.POINTER(FbParams)]),
    "fb_booster_create_sharded": (P, [P, f32p, f32p, C.POINTER(FbParams), C.c_uint64, C.c_uint64, u8p, C.c_int32,
                                      C.c_int32, C.c_uint32]),
    "fb_booster_create_sharded_comm": (P, [P, f32p, f32p, C.POINTER(FbParams), C.c_uint64, C.c_uint64, P,
                                           C.c_int32, C.c_int32]),
    "fbgpu_comm_begin": (C.c_int, [u8p, C.c_int32, C.c_int32, C.c_int32, C.c_uint32, C.POINTER(P)]),
    "fbgpu_comm_free": (None, [P]),
    "fbgpu_comm_usable": (C.c_int32, [P]),
    "fbgpu_quantizer_scales": (C.c_int, [C.c_int32, f32p, C.c_uint64, C.c_uint64, C.POINTER(C.c_double)]),
    "fbgpu_quantizer_scale_digest": (C.c_uint64, [C.c_uint32, C.c_uint32, C.c_uint64]),
    "fbgpu_comm_abort": (None, [P]),
    "fbgpu_ctx_adopt_comm": (C.c_int, [P, P]),
    "fb_booster_free": (None, [P]),
    "fb_booster_update": (C.c_int32, [P, C.c_uint32]),
    "fb_booster_timing": (None, [P, f64p]),
    "fb_booster_collective_ms": (C.c_double, [P]),
    "fb_booster_hist_updates": (C.c_double, [P]),
    "fb_booster_set_stats": (None, [P, C.c_int32]),
    "fb_booster_model": (P, [P]),
    "fb_booster_margins": (C.c_int32, [P, f32p]),
    "fb_train": (P, [f32p, C.c_uint64, C.c_uint32, f32p, f32p, u8p, C.POINTER(FbParams), C.c_uint32]),
    "fb_model_free": (None, [P]),
    "fb_model_num_trees": (C.c_uint32, [P]),
    "fb_model_num_features": (C.c_uint32, [P]),
    "fb_model_base_margin": (C.c_float, [P]),
    "fb_model_json": (C.c_int64, [P, C.c_char_p, C.c_int64]),
    "fb_model_node_cats": (C.c_int64, [P, C.c_uint32, C.c_uint32, u32p, C.c_uint32]),
    "fb_model_tree": (C.c_int64, [P, C.c_uint32, i32p, i32p, u32p, f32p, u8p, f32p, u8p, f32p, f32p, u32p]),
    "fb_model_create": (P, [C.c_uint32, C.c_int32, C.c_float, C.c_float, C.c_uint32, f32p, u8p, C.c_uint32, u32p,
                            i32p, i32p, u32p, f32p, u8p, f32p, f32p, f32p, u8p, u32p, u32p, u32p, C.c_uint64]),
    "fb_model_predict": (C.c_int32, [P, f32p, C.c_uint64, f32p, C.c_int32]),
    "fb_model_num_outputs": (C.c_uint32, [P]),
    "fb_model_transform": (C.c_int32, [P, f32p, C.c_uint64, f32p]),
    "fb_model_shap": (C.c_int32, [P, f32p, C.c_uint64, f32p, C.c_int32]),
    "fb_model_explain": (C.c_int32, [P, C.c_int32, f32p, C.c_uint64, f32p, C.c_int32]),
    "fb_model_device": (P, [P, C.c_int32]),
}

_lib = None


def load():
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m ferrisboost_b200.build` "
            "(this package has no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def ptr(a, ctype):
    return None if a is None else a.ctypes.data_as(C.POINTER(ctype))
