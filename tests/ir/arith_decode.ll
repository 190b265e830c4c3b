; arith_decode.ll -- linear contraction over contiguous KV, one CTA per
; request (task axis ctaid.x): out[req * 64 + d] = sum_t kv[(req * nt + t) * 64 + d] * w[t].
; The KV address is an affine function of the loop's canonical induction
; variable (no index loaded in the loop): an arithmetic stream, the case where
; the urgent policy tier can prefetch a fixed distance ahead.
target datalayout = "e-p:64:64:64-i1:8:8-i8:8:8-i16:16:16-i32:32:32-i64:64:64-f32:32:32-f64:64:64-v16:16:16-v32:32:32-v64:64:64-v128:128:128-n16:32:64"
target triple = "nvptx64-nvidia-cuda"

@__sched_task_order = addrspace(1) externally_initialized global ptr null, align 8
@__sched_ctrl = addrspace(1) externally_initialized global ptr null, align 8
@__sched_timer = addrspace(1) externally_initialized global ptr null, align 8

declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
declare i32 @llvm.nvvm.read.ptx.sreg.tid.x()

define ptx_kernel void @arith_decode(ptr %kv, ptr %w, ptr %out, i32 %nt) {
entry:
  %req = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
  %d = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()
  %row = mul i32 %req, %nt
  br label %loop

loop:
  %i = phi i32 [ 0, %entry ], [ %i.next, %loop ]
  %acc = phi float [ 0.000000e+00, %entry ], [ %acc.next, %loop ]
  %tok = add i32 %row, %i
  %base = mul i32 %tok, 64
  %off = add i32 %base, %d
  %off64 = sext i32 %off to i64
  %kv.gep = getelementptr float, ptr %kv, i64 %off64
  %v = load float, ptr %kv.gep, align 4
  %w.gep = getelementptr float, ptr %w, i32 %i
  %wv = load float, ptr %w.gep, align 4
  %acc.next = call float @llvm.fma.f32(float %v, float %wv, float %acc)
  %i.next = add i32 %i, 1
  %done = icmp eq i32 %i.next, %nt
  br i1 %done, label %exit, label %loop

exit:
  %o.idx0 = mul i32 %req, 64
  %o.idx = add i32 %o.idx0, %d
  %o.gep = getelementptr float, ptr %out, i32 %o.idx
  store float %acc.next, ptr %o.gep, align 4
  ret void
}

declare float @llvm.fma.f32(float, float, float)
