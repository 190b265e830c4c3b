; paged_linear_shuffled.ll -- the paged linear contraction of paged_linear.ll
; with its loop laid out the way a compiler may emit it: the latch block
; comes before the header in the text, the body is split over two blocks,
; the exit block sits between them, and the induction variable's phi lists
; the back edge first and steps with `add nuw nsw i32 1, %i`. A weaver that
; finds loops by block order or matches the phi's text does not see this
; loop; one that computes dominators and natural loops does.
; out[req * 64 + d] = sum_b kv[(bt[req * nb + b] * 64) + d] * w[b]
target datalayout = "e-p:64:64:64-i1:8:8-i8:8:8-i16:16:16-i32:32:32-i64:64:64-f32:32:32-f64:64:64-v16:16:16-v32:32:32-v64:64:64-v128:128:128-n16:32:64"
target triple = "nvptx64-nvidia-cuda"

@__sched_task_order = addrspace(1) externally_initialized global ptr null, align 8
@__sched_ctrl = addrspace(1) externally_initialized global ptr null, align 8
@__sched_timer = addrspace(1) externally_initialized global ptr null, align 8

declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
declare i32 @llvm.nvvm.read.ptx.sreg.tid.x()

define ptx_kernel void @paged_linear_shuffled(ptr %kv, ptr %bt, ptr %w, ptr %out, i32 %nb) {
entry:
  %req = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
  %d = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()
  %row = mul i32 %req, %nb
  br label %head

latch:
  %wv = load float, ptr %w.gep, align 4
  %acc.next = call float @llvm.fma.f32(float %v, float %wv, float %acc)
  %i.next = add nuw nsw i32 1, %i
  %done = icmp eq i32 %i.next, %nb
  br i1 %done, label %exit, label %head

exit:
  %o.idx0 = mul i32 %req, 64
  %o.idx = add i32 %o.idx0, %d
  %o.gep = getelementptr float, ptr %out, i32 %o.idx
  store float %acc.next, ptr %o.gep, align 4
  ret void

head:
  %acc = phi float [ %acc.next, %latch ], [ 0.000000e+00, %entry ]
  %i = phi i32 [ %i.next, %latch ], [ 0, %entry ]
  %bt.idx = add i32 %row, %i
  %bt.gep = getelementptr i32, ptr %bt, i32 %bt.idx
  %page = load i32, ptr %bt.gep, align 4
  %base = mul i32 %page, 64
  %off = add i32 %base, %d
  %kv.gep = getelementptr float, ptr %kv, i32 %off
  %v = load float, ptr %kv.gep, align 4
  %w.gep = getelementptr float, ptr %w, i32 %i
  br label %latch
}

declare float @llvm.fma.f32(float, float, float)
