; async_copy.ll -- a contraction that stages its stream through shared memory
; with cp.async (the pattern of FlashInfer's KV loads): per iteration i, thread
; t copies src[(req * n + i) * 64 + t] into smem[t] with cp.async, waits, and
; accumulates it. The global source is affine in the canonical IV %i.
target datalayout = "e-p:64:64:64-i1:8:8-i8:8:8-i16:16:16-i32:32:32-i64:64:64-f32:32:32-f64:64:64-v16:16:16-v32:32:32-v64:64:64-v128:128:128-n16:32:64"
target triple = "nvptx64-nvidia-cuda"

@__sched_task_order = addrspace(1) externally_initialized global ptr null, align 8
@__sched_ctrl = addrspace(1) externally_initialized global ptr null, align 8
@__sched_timer = addrspace(1) externally_initialized global ptr null, align 8
@smem = internal addrspace(3) global [64 x float] undef, align 16

declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
declare i32 @llvm.nvvm.read.ptx.sreg.tid.x()

define ptx_kernel void @async_copy(ptr addrspace(1) %src, ptr %out, i32 %n) {
entry:
  %req = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
  %t = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()
  %row = mul i32 %req, %n
  %sh = getelementptr [64 x float], ptr addrspace(3) @smem, i32 0, i32 %t
  %sa = ptrtoint ptr addrspace(3) %sh to i32
  br label %loop

loop:
  %i = phi i32 [ 0, %entry ], [ %i.next, %loop ]
  %acc = phi float [ 0.000000e+00, %entry ], [ %acc.next, %loop ]
  %tok = add i32 %row, %i
  %e0 = mul i32 %tok, 64
  %e = add i32 %e0, %t
  %e64 = sext i32 %e to i64
  %g = getelementptr float, ptr addrspace(1) %src, i64 %e64
  call void asm sideeffect "cp.async.ca.shared.global [$0], [$1], 4;", "r,l,~{memory}"(i32 %sa, ptr addrspace(1) %g)
  call void asm sideeffect "cp.async.wait_all;", "~{memory}"()
  %v = load float, ptr addrspace(3) %sh, align 4
  %acc.next = fadd float %acc, %v
  %i.next = add i32 %i, 1
  %done = icmp eq i32 %i.next, %n
  br i1 %done, label %exit, label %loop

exit:
  %o0 = mul i32 %req, 64
  %o = add i32 %o0, %t
  %og = getelementptr float, ptr %out, i32 %o
  store float %acc.next, ptr %og, align 4
  ret void
}
