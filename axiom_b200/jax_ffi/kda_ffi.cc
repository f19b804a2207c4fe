// XLA FFI handlers over the KDA C ABI, for registering the B200 kernels with
// JAX (jax.ffi) as the reference's operator boundary expects: cc_scan's forward
// and backward rules (net/kernels/kda_cc_fused_persist.py:874-932) and the
// decode step (_delta_step, net/kda.py:298-310).
//
// Not part of the library build: it needs the XLA FFI headers that ship inside
// jaxlib (python -c "import jax.ffi; print(jax.ffi.include_dir())"), which this
// build environment does not have.  A maintainer compiles it with
//
//   g++ -std=c++17 -O2 -shared -fPIC -I$(python -c 'import jax.ffi; print(jax.ffi.include_dir())') \
//       -I<repo>/include -I/usr/local/cuda/include kda_ffi.cc -L<repo>/axiom_b200 -lkda_b200 \
//       -Wl,-rpath,<repo>/axiom_b200 -o libkda_ffi.so
//
// and registers the handlers from Python (cc_scan_b200.py beside this file).
// Each handler maps buffer dtypes to KDA_* codes, forwards the device pointers,
// dimensions and the XLA stream to the C ABI, and turns a KDA_ERR_* status into
// an ffi::Error carrying kda_strerror's text (the reference's fail-closed
// contract: nothing falls back).

#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "kda_b200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

int kda_dtype(ffi::DataType t) {
  switch (t) {
    case ffi::DataType::F32: return KDA_F32;
    case ffi::DataType::BF16: return KDA_BF16;
    default: return -1;
  }
}

ffi::Error status(const char* fn, int rc) {
  if (rc == KDA_OK) return ffi::Error::Success();
  return ffi::Error(ffi::ErrorCode::kInvalidArgument, std::string(fn) + ": " + kda_strerror(rc));
}

ffi::Error bad_dtype(const char* fn) {
  return ffi::Error(ffi::ErrorCode::kInvalidArgument,
                    std::string(fn) + ": buffers must be float32 or bfloat16");
}

// q, k, g [B, T, H, dk]; v [B, T, H, dv]; beta [B, T, H]; s0 [B, H, dk, dv] f32.
// Results: o [B, T, H, dv]; s_t [B, H, dk, dv] f32; ckpt u8[kda_ckpt_bytes(...)].
ffi::Error KdaFwd(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v,
                  ffi::AnyBuffer g, ffi::AnyBuffer beta, ffi::Buffer<ffi::F32> s0,
                  ffi::Result<ffi::AnyBuffer> o, ffi::Result<ffi::Buffer<ffi::F32>> s_t,
                  ffi::Result<ffi::AnyBuffer> ckpt, int64_t chunk) {
  const auto d = q.dimensions();
  if (d.size() != 4 || v.dimensions().size() != 4) {
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "kda_fwd: q and v must be [B, T, H, D]");
  }
  const int in_dt = kda_dtype(q.element_type()), o_dt = kda_dtype(o->element_type());
  if (in_dt < 0 || o_dt < 0) return bad_dtype("kda_fwd");
  const int B = static_cast<int>(d[0]), T = static_cast<int>(d[1]), H = static_cast<int>(d[2]);
  const int dk = static_cast<int>(d[3]), dv = static_cast<int>(v.dimensions()[3]);
  const int ck_dt = in_dt;  // the checkpoint is kept in the input precision
  if (ckpt->size_bytes() < kda_ckpt_bytes(B, T, H, dk, dv, static_cast<int>(chunk), in_dt, ck_dt)) {
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "kda_fwd: ckpt result is too small");
  }
  return status("kda_fwd",
                kda_fwd(q.untyped_data(), k.untyped_data(), v.untyped_data(), g.untyped_data(),
                        beta.untyped_data(), s0.typed_data(), o->untyped_data(), s_t->typed_data(),
                        ckpt->untyped_data(), B, T, H, dk, dv, static_cast<int>(chunk), in_dt, o_dt,
                        ck_dt, reinterpret_cast<kda_stream_t>(stream)));
}

// The forward's operands plus the checkpoint, do [B, T, H, dv] and dsT
// [B, H, dk, dv] f32.  Results: dq, dk, dv, dg, dbeta (input dtype), ds0 f32.
// The workspace comes from XLA's scratch allocator.
ffi::Error KdaBwd(cudaStream_t stream, ffi::ScratchAllocator scratch, ffi::AnyBuffer q,
                  ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer g, ffi::AnyBuffer beta,
                  ffi::AnyBuffer ckpt, ffi::AnyBuffer dout, ffi::Buffer<ffi::F32> dsT,
                  ffi::Result<ffi::AnyBuffer> dq, ffi::Result<ffi::AnyBuffer> dk_,
                  ffi::Result<ffi::AnyBuffer> dv_, ffi::Result<ffi::AnyBuffer> dg,
                  ffi::Result<ffi::AnyBuffer> dbeta, ffi::Result<ffi::Buffer<ffi::F32>> ds0,
                  int64_t chunk) {
  const auto d = q.dimensions();
  const int in_dt = kda_dtype(q.element_type()), do_dt = kda_dtype(dout.element_type());
  if (in_dt < 0 || do_dt < 0) return bad_dtype("kda_bwd");
  const int B = static_cast<int>(d[0]), T = static_cast<int>(d[1]), H = static_cast<int>(d[2]);
  const int dk = static_cast<int>(d[3]), dv = static_cast<int>(v.dimensions()[3]);
  const int C = static_cast<int>(chunk);
  const size_t wbytes = kda_bwd_workspace_bytes(B, T, H, dk, dv, C, in_dt);
  void* work = nullptr;
  if (wbytes > 0) {
    auto p = scratch.Allocate(wbytes, 256);
    if (!p.has_value()) {
      return ffi::Error(ffi::ErrorCode::kResourceExhausted, "kda_bwd: scratch allocation failed");
    }
    work = *p;
  }
  return status("kda_bwd",
                kda_bwd(q.untyped_data(), k.untyped_data(), v.untyped_data(), g.untyped_data(),
                        beta.untyped_data(), ckpt.untyped_data(), dout.untyped_data(),
                        dsT.typed_data(), dq->untyped_data(), dk_->untyped_data(),
                        dv_->untyped_data(), dg->untyped_data(), dbeta->untyped_data(),
                        ds0->typed_data(), work, wbytes, B, T, H, dk, dv, C, in_dt, do_dt, in_dt,
                        reinterpret_cast<kda_stream_t>(stream)));
}

// One recurrent token for N = prod(leading dims) states.  s_in [..., dk, dv]
// f32 is aliased to s_out (input_output_aliases={0: 1} on the Python side),
// which the kernel updates in place.
ffi::Error KdaDecode(cudaStream_t stream, ffi::Buffer<ffi::F32> s_in, ffi::AnyBuffer q,
                     ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer g, ffi::AnyBuffer beta,
                     ffi::Result<ffi::AnyBuffer> o, ffi::Result<ffi::Buffer<ffi::F32>> s_out) {
  const auto d = s_in.dimensions();
  if (d.size() < 2) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "kda_decode: S is [..., dk, dv]");
  const int dk = static_cast<int>(d[d.size() - 2]), dv = static_cast<int>(d[d.size() - 1]);
  int64_t N = 1;
  for (size_t i = 0; i + 2 < d.size(); ++i) N *= d[i];
  const int in_dt = kda_dtype(q.element_type()), o_dt = kda_dtype(o->element_type());
  if (in_dt < 0 || o_dt < 0) return bad_dtype("kda_decode");
  if (s_out->typed_data() != s_in.typed_data()) {
    cudaMemcpyAsync(s_out->typed_data(), s_in.typed_data(), s_in.size_bytes(),
                    cudaMemcpyDeviceToDevice, stream);
  }
  return status("kda_decode",
                kda_decode(s_out->typed_data(), q.untyped_data(), k.untyped_data(), v.untyped_data(),
                           g.untyped_data(), beta.untyped_data(), o->untyped_data(),
                           static_cast<int>(N), dk, dv, in_dt, o_dt,
                           reinterpret_cast<kda_stream_t>(stream)));
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(kda_fwd_handler, KdaFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()          // q
                                  .Arg<ffi::AnyBuffer>()          // k
                                  .Arg<ffi::AnyBuffer>()          // v
                                  .Arg<ffi::AnyBuffer>()          // g
                                  .Arg<ffi::AnyBuffer>()          // beta
                                  .Arg<ffi::Buffer<ffi::F32>>()   // s0
                                  .Ret<ffi::AnyBuffer>()          // o
                                  .Ret<ffi::Buffer<ffi::F32>>()   // s_t
                                  .Ret<ffi::AnyBuffer>()          // ckpt
                                  .Attr<int64_t>("chunk"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(kda_bwd_handler, KdaBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Arg<ffi::AnyBuffer>()          // q
                                  .Arg<ffi::AnyBuffer>()          // k
                                  .Arg<ffi::AnyBuffer>()          // v
                                  .Arg<ffi::AnyBuffer>()          // g
                                  .Arg<ffi::AnyBuffer>()          // beta
                                  .Arg<ffi::AnyBuffer>()          // ckpt
                                  .Arg<ffi::AnyBuffer>()          // do
                                  .Arg<ffi::Buffer<ffi::F32>>()   // dsT
                                  .Ret<ffi::AnyBuffer>()          // dq
                                  .Ret<ffi::AnyBuffer>()          // dk
                                  .Ret<ffi::AnyBuffer>()          // dv
                                  .Ret<ffi::AnyBuffer>()          // dg
                                  .Ret<ffi::AnyBuffer>()          // dbeta
                                  .Ret<ffi::Buffer<ffi::F32>>()   // ds0
                                  .Attr<int64_t>("chunk"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(kda_decode_handler, KdaDecode,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()   // S (aliased to the S result)
                                  .Arg<ffi::AnyBuffer>()          // q
                                  .Arg<ffi::AnyBuffer>()          // k
                                  .Arg<ffi::AnyBuffer>()          // v
                                  .Arg<ffi::AnyBuffer>()          // g
                                  .Arg<ffi::AnyBuffer>()          // beta
                                  .Ret<ffi::AnyBuffer>()          // o
                                  .Ret<ffi::Buffer<ffi::F32>>()); // S updated
