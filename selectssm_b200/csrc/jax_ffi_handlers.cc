// XLA FFI handlers that let JAX call the C ABI directly (jax.ffi custom calls).
//
// UNVERIFIED: JAX/jaxlib are not installed where this library is developed,
// so this file is not compiled by the default build.  In an environment with
// jaxlib it is built by selectssm_b200.jax_ffi.build_handlers() against the
// headers of jax.ffi.include_dir() and linked to libselectssm_b200.so.
//
// Each handler replaces one function of the reference's scan path:
//   selectssm_scan_fwd  ssm_chunked_scan / ssm_recursive_scan / ssm_scan forward
//                       (src/selectssm/selectssm.py:37-109,
//                        src/selectssm/ssmrecscan.py:36-88), optionally fused
//                       with softplus(delta + bias), the D skip and the gate
//   selectssm_scan_bwd  the custom-VJP backward (src/selectssm/ssmrecscan.py:111-181)
// Arrays are the reference's channels-last layouts: x, delta, z (B, L, D),
// B, C (B, L, N), A (D, N), D and bias (D,).  Optional operands (D, bias, z)
// are passed as zero-size arrays when absent.  Scratch is an extra u8 result
// sized by ssm_workspace_bytes on the host.

#include <cstdint>

#include "xla/ffi/api/ffi.h"
#include "selectssm_b200.h"

namespace ffi = xla::ffi;

namespace {

int32_t dtype_code(ffi::DataType t) { return t == ffi::DataType::BF16 ? SSM_BF16 : SSM_F32; }

template <typename Buf>
const void* opt(const Buf& b) {
  return b.element_count() ? b.untyped_data() : nullptr;
}

ffi::Error status_error(int st) {
  if (st == SSM_OK) return ffi::Error::Success();
  const ffi::ErrorCode code = (st == SSM_ERR_SHAPE || st == SSM_ERR_DTYPE || st == SSM_ERR_ALIGN)
                                  ? ffi::ErrorCode::kInvalidArgument
                                  : ffi::ErrorCode::kInternal;
  return ffi::Error(code, ssm_strerror(st));
}

void fill_common(ssm_params_t* p, const ffi::AnyBuffer& x, const ffi::AnyBuffer& B, int32_t flags,
                 int32_t gate_act) {
  const auto dims = x.dimensions();
  p->batch = static_cast<int32_t>(dims[0]);
  p->seqlen = static_cast<int32_t>(dims[1]);
  p->dim = static_cast<int32_t>(dims[2]);
  p->dstate = static_cast<int32_t>(B.dimensions()[2]);
  p->dtype = dtype_code(x.element_type());
  p->bc_dtype = dtype_code(B.element_type());
  p->flags = flags;
  p->gate_act = gate_act;
}

ffi::Error ScanFwd(cudaStream_t stream, ffi::AnyBuffer x, ffi::AnyBuffer delta, ffi::Buffer<ffi::F32> A,
                   ffi::AnyBuffer B, ffi::AnyBuffer C, ffi::Buffer<ffi::F32> D, ffi::Buffer<ffi::F32> bias,
                   ffi::AnyBuffer z, ffi::Result<ffi::AnyBuffer> out, ffi::Result<ffi::Buffer<ffi::F32>> states,
                   ffi::Result<ffi::AnyBuffer> workspace, int32_t flags, int32_t gate_act) {
  ssm_params_t p = {};
  fill_common(&p, x, B, flags, gate_act);
  p.u = x.untyped_data();
  p.delta = delta.untyped_data();
  p.A = A.typed_data();
  p.Bm = B.untyped_data();
  p.Cm = C.untyped_data();
  p.D = static_cast<const float*>(opt(D));
  p.delta_bias = static_cast<const float*>(opt(bias));
  p.z = opt(z);
  p.out = out->untyped_data();
  p.states = states->typed_data();
  p.workspace = workspace->untyped_data();
  p.workspace_bytes = workspace->size_bytes();
  return status_error(ssm_fwd(&p, reinterpret_cast<ssm_stream_t>(stream)));
}

ffi::Error ScanBwd(cudaStream_t stream, ffi::AnyBuffer x, ffi::AnyBuffer delta, ffi::Buffer<ffi::F32> A,
                   ffi::AnyBuffer B, ffi::AnyBuffer C, ffi::Buffer<ffi::F32> D, ffi::Buffer<ffi::F32> bias,
                   ffi::AnyBuffer z, ffi::Buffer<ffi::F32> states, ffi::AnyBuffer dout,
                   ffi::Result<ffi::AnyBuffer> dx, ffi::Result<ffi::AnyBuffer> ddelta,
                   ffi::Result<ffi::Buffer<ffi::F32>> dA, ffi::Result<ffi::AnyBuffer> dB,
                   ffi::Result<ffi::AnyBuffer> dC, ffi::Result<ffi::Buffer<ffi::F32>> dD,
                   ffi::Result<ffi::Buffer<ffi::F32>> dbias, ffi::Result<ffi::AnyBuffer> dz,
                   ffi::Result<ffi::AnyBuffer> workspace, int32_t flags, int32_t gate_act) {
  ssm_params_t p = {};
  fill_common(&p, x, B, flags, gate_act);
  p.u = x.untyped_data();
  p.delta = delta.untyped_data();
  p.A = A.typed_data();
  p.Bm = B.untyped_data();
  p.Cm = C.untyped_data();
  p.D = static_cast<const float*>(opt(D));
  p.delta_bias = static_cast<const float*>(opt(bias));
  p.z = opt(z);
  p.states = const_cast<float*>(states.typed_data());
  p.dout = dout.untyped_data();
  p.du = dx->untyped_data();
  p.ddelta = ddelta->untyped_data();
  p.dA = dA->typed_data();
  p.dB = dB->untyped_data();
  p.dC = dC->untyped_data();
  p.dD = dD->element_count() ? dD->typed_data() : nullptr;
  p.ddelta_bias = dbias->element_count() ? dbias->typed_data() : nullptr;
  p.dz = dz->element_count() ? dz->untyped_data() : nullptr;
  p.workspace = workspace->untyped_data();
  p.workspace_bytes = workspace->size_bytes();
  return status_error(ssm_bwd(&p, reinterpret_cast<ssm_stream_t>(stream)));
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(selectssm_scan_fwd, ScanFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()          // x
                                  .Arg<ffi::AnyBuffer>()          // delta
                                  .Arg<ffi::Buffer<ffi::F32>>()   // A
                                  .Arg<ffi::AnyBuffer>()          // B
                                  .Arg<ffi::AnyBuffer>()          // C
                                  .Arg<ffi::Buffer<ffi::F32>>()   // D (or empty)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // delta bias (or empty)
                                  .Arg<ffi::AnyBuffer>()          // z (or empty)
                                  .Ret<ffi::AnyBuffer>()          // out
                                  .Ret<ffi::Buffer<ffi::F32>>()   // states
                                  .Ret<ffi::AnyBuffer>()          // workspace
                                  .Attr<int32_t>("flags")
                                  .Attr<int32_t>("gate_act"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(selectssm_scan_bwd, ScanBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()          // x
                                  .Arg<ffi::AnyBuffer>()          // delta
                                  .Arg<ffi::Buffer<ffi::F32>>()   // A
                                  .Arg<ffi::AnyBuffer>()          // B
                                  .Arg<ffi::AnyBuffer>()          // C
                                  .Arg<ffi::Buffer<ffi::F32>>()   // D (or empty)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // delta bias (or empty)
                                  .Arg<ffi::AnyBuffer>()          // z (or empty)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // states from the forward
                                  .Arg<ffi::AnyBuffer>()          // dout
                                  .Ret<ffi::AnyBuffer>()          // dx
                                  .Ret<ffi::AnyBuffer>()          // ddelta
                                  .Ret<ffi::Buffer<ffi::F32>>()   // dA
                                  .Ret<ffi::AnyBuffer>()          // dB
                                  .Ret<ffi::AnyBuffer>()          // dC
                                  .Ret<ffi::Buffer<ffi::F32>>()   // dD (or empty)
                                  .Ret<ffi::Buffer<ffi::F32>>()   // d delta bias (or empty)
                                  .Ret<ffi::AnyBuffer>()          // dz (or empty)
                                  .Ret<ffi::AnyBuffer>()          // workspace
                                  .Attr<int32_t>("flags")
                                  .Attr<int32_t>("gate_act"));
