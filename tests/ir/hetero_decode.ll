; hetero_decode.ll -- a heterogeneous continuous batch as one kernel: request
; `req` (one CTA, the task axis is ctaid.x) streams nbl[req] KV blocks of 64
; tokens x 128 floats through its block table and contracts them with a
; 64-entry weight vector:
;   out[req * 128 + d] = sum_{b < nbl[req]} sum_{t < 64} kv[(bt[req * bts + b] * 64 + t) * 128 + d] * w[t]
; Thread d owns output element d. Requests differ only in nbl (long and short
; requests), so the step time is decided by how the long ones are placed:
; the shape of jc-su/sched-pass test/hetero_batch.cu (8 long x 32 blocks, 56
; short x 4 blocks, 16 workers), written here as IR for the weaver. The
; outer loop (KV blocks) has the canonical IV that shed truncates.
target datalayout = "e-p:64:64:64-i1:8:8-i8:8:8-i16:16:16-i32:32:32-i64:64:64-f32:32:32-f64:64:64-v16:16:16-v32:32:32-v64:64:64-v128:128:128-n16:32:64"
target triple = "nvptx64-nvidia-cuda"

@__sched_task_order = addrspace(1) externally_initialized global ptr null, align 8
@__sched_ctrl = addrspace(1) externally_initialized global ptr null, align 8
@__sched_timer = addrspace(1) externally_initialized global ptr null, align 8

declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
declare i32 @llvm.nvvm.read.ptx.sreg.tid.x()

define ptx_kernel void @hetero_decode(ptr %kv, ptr %bt, ptr %nbl, ptr %w, ptr %out, i32 %bts) {
entry:
  %req = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
  %d = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()
  %nb.gep = getelementptr i32, ptr %nbl, i32 %req
  %nb = load i32, ptr %nb.gep, align 4
  %row = mul i32 %req, %bts
  %has = icmp sgt i32 %nb, 0
  br i1 %has, label %blk, label %exit

blk:
  %b = phi i32 [ 0, %entry ], [ %b.next, %latch ]
  %acc = phi float [ 0.000000e+00, %entry ], [ %acc.t, %latch ]
  %bt.idx = add i32 %row, %b
  %bt.gep = getelementptr i32, ptr %bt, i32 %bt.idx
  %page = load i32, ptr %bt.gep, align 4
  %pbase = mul i32 %page, 8192
  br label %tok

tok:
  %t = phi i32 [ 0, %blk ], [ %t.next, %tok ]
  %acc.i = phi float [ %acc, %blk ], [ %acc.f, %tok ]
  %trow = mul i32 %t, 128
  %o1 = add i32 %pbase, %trow
  %o2 = add i32 %o1, %d
  %kv.gep = getelementptr float, ptr %kv, i32 %o2
  %v = load float, ptr %kv.gep, align 4
  %w.gep = getelementptr float, ptr %w, i32 %t
  %wv = load float, ptr %w.gep, align 4
  %acc.f = call float @llvm.fma.f32(float %v, float %wv, float %acc.i)
  %t.next = add i32 %t, 1
  %tdone = icmp eq i32 %t.next, 64
  br i1 %tdone, label %latch, label %tok

latch:
  %acc.t = phi float [ %acc.f, %tok ]
  %b.next = add i32 %b, 1
  %bdone = icmp eq i32 %b.next, %nb
  br i1 %bdone, label %exit, label %blk

exit:
  %res = phi float [ 0.000000e+00, %entry ], [ %acc.t, %latch ]
  %o.idx0 = mul i32 %req, 128
  %o.idx = add i32 %o.idx0, %d
  %o.gep = getelementptr float, ptr %out, i32 %o.idx
  store float %res, ptr %o.gep, align 4
  ret void
}

declare float @llvm.fma.f32(float, float, float)
