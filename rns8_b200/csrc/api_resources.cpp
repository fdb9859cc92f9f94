// Contexts, resident matrices, workspaces and their introspection.
//
// Reference behaviour followed here:
//   src/core/api_context.cpp:7-225            context creation (device_id < 0 -> 0), device info
//   src/core/api_matrix_public_api.inc:1-183  matrix creation, instance ids, storage info
//   src/core/api_workspace_public_api.inc     workspace bound to a plan
// A context owns one CUDA stream on one device; every call on it is
// synchronous (it ends with a stream synchronisation), as in the reference.
#include <cstring>

#include "api_internal.hpp"

namespace rns8host {

rns8_status DevBuf::ensure(int dev, uint64_t need) {
  if (ptr && bytes >= need && device == dev) return RNS8_SUCCESS;
  release();
  if (need == 0) return RNS8_SUCCESS;
  void* p = nullptr;
  DeviceScope scope(dev);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  const cudaError_t e = cudaMalloc(&p, need);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return RNS8_BACKEND_FAILURE;
  }
  ptr = p;
  bytes = need;
  device = dev;
  return RNS8_SUCCESS;
}

void DevBuf::release() {
  if (ptr) {
    DeviceScope scope(device);
    cudaFree(ptr);
  }
  ptr = nullptr;
  bytes = 0;
  device = -1;
}

}  // namespace rns8host

using namespace rns8host;

extern "C" rns8_status rns8_create_context(int device_id, const rns8_context_options* options, rns8_context** out) {
  return guard([&]() -> rns8_status {
    if (!out) return RNS8_INVALID_ARGUMENT;
    *out = nullptr;
    rns8_backend_kind requested = RNS8_BACKEND_AUTO;
    if (options) {
      if (!valid_abi(options->struct_size, options->abi_version, sizeof(*options))) return RNS8_INVALID_ARGUMENT;
      if (options->flags != 0) return RNS8_INVALID_ARGUMENT;
      requested = options->requested_backend;
    }
    // This library is the CUDA sm_100a backend only: no CPU fallback.
    if (!backend_request_ok(requested)) return RNS8_UNSUPPORTED_BACKEND;
    const int dev = device_id < 0 ? 0 : device_id;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
      (void)cudaGetLastError();
      return RNS8_UNSUPPORTED_BACKEND;
    }
    if (dev >= count) return RNS8_INVALID_ARGUMENT;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return RNS8_BACKEND_FAILURE;
    if (prop.major != 10 || prop.minor != 0) return RNS8_UNSUPPORTED_ARCH;  // kernels are built for sm_100a only
    DeviceScope scope(dev);
    if (!scope.ok) return RNS8_BACKEND_FAILURE;
    auto* ctx = new (std::nothrow) rns8_context();
    if (!ctx) return RNS8_INTERNAL_ERROR;
    ctx->device_id = dev;
    ctx->sm_count = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->out_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&ctx->dev_status), 4 * sizeof(uint32_t)) != cudaSuccess) {
      if (ctx->stream) cudaStreamDestroy(ctx->stream);
      if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
      if (ctx->out_stream) cudaStreamDestroy(ctx->out_stream);
      delete ctx;
      return RNS8_BACKEND_FAILURE;
    }
    int rt = 0, drv = 0;
    cudaRuntimeGetVersion(&rt);
    cudaDriverGetVersion(&drv);
    rns8_device_info& info = ctx->info;
    info.struct_size = sizeof(info);
    info.abi_version = RNS8_ABI_VERSION;
    info.backend = RNS8_BACKEND_CUDA_SM100;
    info.device_id = dev;
    info.hip_available = 1;
    info.hip_runtime_version = static_cast<uint32_t>(rt);
    info.hip_driver_version = static_cast<uint32_t>(drv);
    info.global_mem_bytes = prop.totalGlobalMem;
    set_text(info.name, sizeof(info.name), prop.name);
    set_text(info.gcn_arch, sizeof(info.gcn_arch), "sm_100a");
    set_text(info.detail, sizeof(info.detail),
             "CUDA sm_100a backend: tcgen05 int8 plane GEMM, " + std::to_string(prop.multiProcessorCount) + " SMs");
    *out = ctx;
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_destroy_context(rns8_context* ctx) {
  if (!ctx) return RNS8_SUCCESS;
  DeviceScope scope(ctx->device_id);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->copy_stream) cudaStreamSynchronize(ctx->copy_stream);
  if (ctx->out_stream) cudaStreamSynchronize(ctx->out_stream);
  ctx->oneshot_arena.release();
  ctx->admission.release();
  if (ctx->dev_status) cudaFree(ctx->dev_status);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
  if (ctx->out_stream) cudaStreamDestroy(ctx->out_stream);
  delete ctx;
  return RNS8_SUCCESS;
}

extern "C" rns8_status rns8_get_device_info(rns8_context* ctx, rns8_device_info* out) {
  return guard([&]() -> rns8_status {
    if (!ctx || !out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = ctx->info;
    out->struct_size = ss;
    out->abi_version = av;
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_get_backend_capability_info(rns8_backend_kind backend, rns8_backend_capability_info* out) {
  return guard([&]() -> rns8_status {
    if (!out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    if (static_cast<uint32_t>(backend) > RNS8_BACKEND_CUDA_SM100) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = {};
    out->struct_size = ss;
    out->abi_version = av;
    out->backend = backend;
    const bool ours = backend == RNS8_BACKEND_CUDA_SM100 || backend == RNS8_BACKEND_AUTO;
    int count = 0;
    const bool device = cudaGetDeviceCount(&count) == cudaSuccess && count > 0;
    if (!device) (void)cudaGetLastError();
    out->is_accelerator = ours ? 1u : 0u;
    out->is_available = (ours && device) ? 1u : 0u;
    out->is_matrix_engine_backend = ours ? 1u : 0u;
    out->supports_bounded_rns = ours ? 1u : 0u;
    out->supports_exact_wide_rns = ours ? 1u : 0u;
    out->supports_finite_u8 = ours ? 1u : 0u;
    out->supports_wrap64 = ours ? 1u : 0u;
    out->requires_feature_detection = ours ? 1u : 0u;
    out->compiled_kernel_available = ours ? 1u : 0u;
    out->exact_differential_validated = ours ? 1u : 0u;
    set_text(out->backend_name, sizeof(out->backend_name), ours ? "cuda_sm100" : "not_built");
    set_text(out->selected_kernel, sizeof(out->selected_kernel),
             ours ? "sm100a_tcgen05_i8_plane_gemm_128x256x128_modm_epilogue" : "");
    set_text(out->library_name, sizeof(out->library_name), "rns8_b200");
    set_text(out->library_version, sizeof(out->library_version), "1");
    set_text(out->epilogue_mode, sizeof(out->epilogue_mode), ours ? "int32_tmem_to_centered_residue_mulhi" : "");
    set_text(out->isa_evidence, sizeof(out->isa_evidence), ours ? "tcgen05.mma.kind::i8" : "");
    set_text(out->status, sizeof(out->status),
             ours ? (device ? "available" : "no CUDA device") : "backend not provided by this library");
    return RNS8_SUCCESS;
  });
}

// ---- matrices --------------------------------------------------------------------
extern "C" rns8_status rns8_create_matrix(rns8_context* ctx, const rns8_matrix_desc* desc, rns8_matrix** out) {
  return guard([&]() -> rns8_status {
    if (!ctx || !desc || !out) return RNS8_INVALID_ARGUMENT;
    *out = nullptr;
    if (!valid_abi(desc->struct_size, desc->abi_version, sizeof(*desc))) return RNS8_INVALID_ARGUMENT;
    const uint32_t prefix = desc->max_prefix == 0 ? default_prefix_for_semantics(desc->semantics) : desc->max_prefix;
    const rns8_status v = validate_matrix_desc(*desc, prefix);
    if (v != RNS8_SUCCESS) return v;
    const bool wrap = desc->semantics == RNS8_WRAP_U64_MOD_2_64;
    // Residue planes; finite storage has one; wrap64 keeps eight byte planes.
    const uint64_t planes = wrap ? 8 : (uses_finite_storage(desc->semantics) ? 1 : prefix);
    const uint64_t cells = static_cast<uint64_t>(desc->rows) * static_cast<uint64_t>(desc->cols);
    if (desc->cols != 0 && static_cast<uint64_t>(desc->rows) > UINT64_MAX / static_cast<uint64_t>(desc->cols))
      return RNS8_RANGE_ERROR;
    if (cells > UINT64_MAX / planes) return RNS8_RANGE_ERROR;
    auto* mtx = new (std::nothrow) rns8_matrix();
    if (!mtx) return RNS8_INTERNAL_ERROR;
    mtx->id = next_matrix_id();
    mtx->desc = *desc;
    mtx->desc.struct_size = sizeof(rns8_matrix_desc);
    mtx->desc.max_prefix = prefix;
    if (mtx->desc.logical_ld == 0) mtx->desc.logical_ld = mtx->desc.cols;
    if (mtx->desc.tile_m == 0) mtx->desc.tile_m = 128;
    if (mtx->desc.tile_n == 0) mtx->desc.tile_n = 128;
    mtx->prefix = prefix;
    mtx->device_id = ctx->device_id;
    mtx->residue_bytes = cells * planes;
    DeviceScope scope(ctx->device_id);
    if (!scope.ok || cudaMalloc(reinterpret_cast<void**>(&mtx->residues), mtx->residue_bytes) != cudaSuccess) {
      (void)cudaGetLastError();
      delete mtx;
      return RNS8_BACKEND_FAILURE;
    }
    // A fresh matrix is logically zero: zero residues represent the value 0.
    if (cudaMemsetAsync(mtx->residues, 0, mtx->residue_bytes, ctx->stream) != cudaSuccess ||
        cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
      cudaFree(mtx->residues);
      delete mtx;
      return RNS8_BACKEND_FAILURE;
    }
    mtx->device_current = false;
    if (exact_wide(desc->semantics)) {
      mtx->exact_range_prefix = 0;
    }
    *out = mtx;
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_destroy_matrix(rns8_matrix* matrix) {
  if (!matrix) return RNS8_SUCCESS;
  DeviceScope scope(matrix->device_id);
  if (matrix->residues) cudaFree(matrix->residues);
  delete matrix;
  return RNS8_SUCCESS;
}

extern "C" rns8_status rns8_get_matrix_storage_info(const rns8_matrix* m, rns8_matrix_storage_info* out) {
  return guard([&]() -> rns8_status {
    if (!m || !out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = {};
    out->struct_size = ss;
    out->abi_version = av;
    out->backend = m->backend;
    out->semantics = m->desc.semantics;
    out->logical_layout = m->desc.logical_layout;
    out->bound_kind = m->desc.bound_kind;
    out->rows = m->desc.rows;
    out->cols = m->desc.cols;
    out->logical_ld = m->desc.logical_ld;
    out->max_prefix = m->prefix;
    out->finite_modulus = m->finite_modulus;
    out->matrix_instance_id = m->id;
    out->source_version = m->source_version;
    out->host_residues_current = 0;
    out->hip_device_id = m->device_id;
    // Storage scope and layout identifiers are the reference's contract names
    // for device storage of these layouts (api_plan_workspace_packing.inc:227-260).
    set_text(out->storage_scope, sizeof(out->storage_scope), "device_resident_storage");
    if (m->desc.semantics == RNS8_WRAP_U64_MOD_2_64) {
      out->device_byte_limbs_current = m->device_current ? 1u : 0u;
      out->uses_byte_limb_storage = 1;
      out->device_byte_limb_bytes = m->residue_bytes;
      set_text(out->storage_scope, sizeof(out->storage_scope), "device_byte_limb_storage");
      set_text(out->layout_version, sizeof(out->layout_version), "wrap64_byte_limb_v1");
      set_text(out->detail, sizeof(out->detail), "eight unsigned byte planes on device " + std::to_string(m->device_id));
      return RNS8_SUCCESS;
    }
    out->device_residues_current = m->device_current ? 1u : 0u;
    out->uses_residue_storage = 1;
    out->device_residue_bytes = m->residue_bytes;
    set_text(out->layout_version, sizeof(out->layout_version),
             uses_finite_storage(m->desc.semantics) ? "finite_u8_centered_residue_v1" : "rns_centered_residue_planes_v1");
    set_text(out->detail, sizeof(out->detail), "centered int8 residue planes on device " + std::to_string(m->device_id));
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_get_resident_lifetime_info(const rns8_matrix* matrix, const rns8_plan* plan,
                                                       const rns8_workspace* workspace,
                                                       rns8_resident_matrix_role role,
                                                       rns8_resident_lifetime_info* out) {
  return guard([&]() -> rns8_status {
    if (!matrix || !out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    if (workspace && !plan) return RNS8_INVALID_ARGUMENT;
    if (static_cast<uint32_t>(role) > RNS8_RESIDENT_MATRIX_ROLE_C) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = {};
    out->struct_size = ss;
    out->abi_version = av;
    out->backend = matrix->backend;
    out->semantics = matrix->desc.semantics;
    out->logical_layout = matrix->desc.logical_layout;
    out->bound_kind = matrix->desc.bound_kind;
    out->matrix_role = role;
    const bool finite = uses_finite_storage(matrix->desc.semantics);
    const bool wrap = matrix->desc.semantics == RNS8_WRAP_U64_MOD_2_64;
    out->current_output_domain = wrap ? RNS8_OUTPUT_DOMAIN_WRAP64_BYTE_LIMB
                                      : (finite ? RNS8_OUTPUT_DOMAIN_FINITE_U8 : RNS8_OUTPUT_DOMAIN_RNS_RESIDUE);
    out->rows = matrix->desc.rows;
    out->cols = matrix->desc.cols;
    out->logical_ld = matrix->desc.logical_ld;
    out->max_prefix = matrix->prefix;
    out->finite_modulus = matrix->finite_modulus;
    out->source_version = matrix->source_version;
    out->source_version_valid = matrix->source_version != 0 ? 1u : 0u;
    out->device_current = matrix->device_current ? 1u : 0u;
    out->device_resident = 1;
    out->hip_device_id = matrix->device_id;
    if (plan) {
      out->plan_fingerprint = plan->fingerprint;
      out->plan_binding_available = 1;
      out->plan_binding_matches = plan->desc.semantics == matrix->desc.semantics ? 1u : 0u;
      out->device_id_matches = plan->device_id == matrix->device_id ? 1u : 0u;
    }
    if (workspace) {
      out->workspace_fingerprint = workspace->plan_fingerprint;
      out->workspace_binding_available = 1;
      out->workspace_identity_matches = workspace->plan_fingerprint == plan->fingerprint ? 1u : 0u;
      out->workspace_binding_matches = out->workspace_identity_matches;
      out->workspace_backend_matches = 1;
      out->workspace_schedule_matches = out->workspace_identity_matches;
    }
    out->can_feed_rns_gemm = (!finite && !wrap && matrix->device_current) ? 1u : 0u;
    out->can_feed_final_export = matrix->device_current ? 1u : 0u;
    set_text(out->current_domain, sizeof(out->current_domain),
             wrap ? "wrap64_byte_limb" : (finite ? "finite_u8" : "rns_residue"));
    const char* names[] = {"unknown", "a", "b", "c"};
    set_text(out->matrix_role_name, sizeof(out->matrix_role_name), names[static_cast<uint32_t>(role)]);
    set_text(out->source_version_policy, sizeof(out->source_version_policy), "nonzero_version_elides_repack");
    return RNS8_SUCCESS;
  });
}

// ---- workspaces ----------------------------------------------------------------
extern "C" rns8_status rns8_create_workspace(rns8_context* ctx, const rns8_plan* plan, rns8_workspace** out) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !out) return RNS8_INVALID_ARGUMENT;
    *out = nullptr;
    if (plan->device_id != ctx->device_id) return RNS8_INVALID_ARGUMENT;
    auto* ws = new (std::nothrow) rns8_workspace();
    if (!ws) return RNS8_INTERNAL_ERROR;
    ws->device_id = ctx->device_id;
    ws->plan_fingerprint = plan->fingerprint;
    ws->semantics = plan->desc.semantics;
    ws->bound_kind = plan->desc.bound_kind;
    ws->m = plan->desc.m;
    ws->n = plan->desc.n;
    ws->k = plan->desc.k;
    ws->prefix = plan->prefix;
    *out = ws;
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_destroy_workspace(rns8_workspace* workspace) {
  delete workspace;
  return RNS8_SUCCESS;
}
