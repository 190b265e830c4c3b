; softmax_decode.ll -- paged online-softmax decode attention, fp32.
; One CTA per request (ctaid.x = task), one thread per query head (tid.x);
; the G query heads of a request share one KV head. head_dim 64, page 16.
;   q   [req][G][64]        kc, vc [page][16][64]      bt [req][maxp]
;   len [req]               out [req][G][64]
; For each token t < len: s = scale * dot(q, k_t); online softmax (running
; max m via llvm.maxnum, weights via llvm.exp2 in the log2 domain), then the
; accumulator o += p * v_t. The token loop's induction variable %t is the
; canonical IV the shed lever masks on (tokens >= tau drop out of the softmax).
target datalayout = "e-p:64:64:64-i1:8:8-i8:8:8-i16:16:16-i32:32:32-i64:64:64-f32:32:32-f64:64:64-v16:16:16-v32:32:32-v64:64:64-v128:128:128-n16:32:64"
target triple = "nvptx64-nvidia-cuda"

@__sched_task_order = addrspace(1) externally_initialized global ptr null, align 8
@__sched_ctrl = addrspace(1) externally_initialized global ptr null, align 8
@__sched_timer = addrspace(1) externally_initialized global ptr null, align 8

declare i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
declare i32 @llvm.nvvm.read.ptx.sreg.tid.x()
declare float @llvm.maxnum.f32(float, float)
declare float @llvm.exp2.f32(float)

define ptx_kernel void @softmax_decode(ptr %q, ptr %kc, ptr %vc, ptr %bt, ptr %len, ptr %out, ptr %acc, i32 %maxp, i32 %G, float %scale) {
entry:
  %req = call i32 @llvm.nvvm.read.ptx.sreg.ctaid.x()
  %h = call i32 @llvm.nvvm.read.ptx.sreg.tid.x()
  %len.gep = getelementptr i32, ptr %len, i32 %req
  %n = load i32, ptr %len.gep, align 4
  %rg = mul i32 %req, %G
  %qh = add i32 %rg, %h
  %qbase = mul i32 %qh, 64
  %btrow = mul i32 %req, %maxp
  br label %zero

zero:                                   ; acc[qh][0..64) = 0
  %z = phi i32 [ 0, %entry ], [ %z.next, %zero ]
  %zi = add i32 %qbase, %z
  %z.gep = getelementptr float, ptr %acc, i32 %zi
  store float 0.000000e+00, ptr %z.gep, align 4
  %z.next = add i32 %z, 1
  %z.done = icmp eq i32 %z.next, 64
  br i1 %z.done, label %tok.pre, label %zero

tok.pre:
  %any = icmp sgt i32 %n, 0
  br i1 %any, label %tok, label %fin

tok:
  %t = phi i32 [ 0, %tok.pre ], [ %t.next, %tok.latch ]
  %m = phi float [ 0xFFF0000000000000, %tok.pre ], [ %m.next, %tok.latch ]
  %l = phi float [ 0.000000e+00, %tok.pre ], [ %l.next, %tok.latch ]
  %pidx = lshr i32 %t, 4
  %slot = and i32 %t, 15
  %bt.i = add i32 %btrow, %pidx
  %bt.gep = getelementptr i32, ptr %bt, i32 %bt.i
  %page = load i32, ptr %bt.gep, align 4
  %p16 = mul i32 %page, 16
  %row = add i32 %p16, %slot
  %kvbase = mul i32 %row, 64
  br label %dot

dot:
  %d = phi i32 [ 0, %tok ], [ %d.next, %dot ]
  %s.acc = phi float [ 0.000000e+00, %tok ], [ %s.next, %dot ]
  %qi = add i32 %qbase, %d
  %q.gep = getelementptr float, ptr %q, i32 %qi
  %qv = load float, ptr %q.gep, align 4
  %ki = add i32 %kvbase, %d
  %k.gep = getelementptr float, ptr %kc, i32 %ki
  %kv = load float, ptr %k.gep, align 4
  %s.next = call float @llvm.fma.f32(float %qv, float %kv, float %s.acc)
  %d.next = add i32 %d, 1
  %d.done = icmp eq i32 %d.next, 64
  br i1 %d.done, label %upd, label %dot

upd:
  %s = fmul float %s.next, %scale
  %m.next = call float @llvm.maxnum.f32(float %m, float %s)
  %dm = fsub float %m, %m.next
  %alpha = call float @llvm.exp2.f32(float %dm)
  %ds = fsub float %s, %m.next
  %p = call float @llvm.exp2.f32(float %ds)
  %la = fmul float %l, %alpha
  %l.next = fadd float %la, %p
  br label %pv

pv:
  %e = phi i32 [ 0, %upd ], [ %e.next, %pv ]
  %ai = add i32 %qbase, %e
  %a.gep = getelementptr float, ptr %acc, i32 %ai
  %av = load float, ptr %a.gep, align 4
  %vi = add i32 %kvbase, %e
  %v.gep = getelementptr float, ptr %vc, i32 %vi
  %vv = load float, ptr %v.gep, align 4
  %pvv = fmul float %p, %vv
  %as = fmul float %av, %alpha
  %an = fadd float %as, %pvv
  store float %an, ptr %a.gep, align 4
  %e.next = add i32 %e, 1
  %e.done = icmp eq i32 %e.next, 64
  br i1 %e.done, label %tok.latch, label %pv

tok.latch:
  %t.next = add i32 %t, 1
  %t.done = icmp eq i32 %t.next, %n
  br i1 %t.done, label %fin.pre, label %tok

fin.pre:
  %lf = phi float [ %l.next, %tok.latch ]
  br label %fin

fin:
  %lsum = phi float [ 0.000000e+00, %tok.pre ], [ %lf, %fin.pre ]
  %has = fcmp ogt float %lsum, 0.000000e+00
  %inv = fdiv float 1.000000e+00, %lsum
  %invs = select i1 %has, float %inv, float 0.000000e+00
  br label %wr

wr:
  %o = phi i32 [ 0, %fin ], [ %o.next, %wr ]
  %oi = add i32 %qbase, %o
  %oa.gep = getelementptr float, ptr %acc, i32 %oi
  %oa = load float, ptr %oa.gep, align 4
  %ov = fmul float %oa, %invs
  %oo.gep = getelementptr float, ptr %out, i32 %oi
  store float %ov, ptr %oo.gep, align 4
  %o.next = add i32 %o, 1
  %o.done = icmp eq i32 %o.next, 64
  br i1 %o.done, label %ret, label %wr

ret:
  ret void
}

declare float @llvm.fma.f32(float, float, float)
