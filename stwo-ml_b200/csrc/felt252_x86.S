/*
 * x86-64 (BMI2 + ADX) Montgomery multiplication for the Stark prime
 * p = 2^251 + 17*2^192 + 1 = [1, 0, 0, 0x0800000000000011] (64-bit limbs),
 * R = 2^256:  r = a * b / R mod p  for a, b < p.
 *
 * void zk_felt_mont_mul_adx(uint64_t r[4], const uint64_t a[4], const uint64_t b[4]);
 *
 * 4x4 schoolbook product with the two ADX carry chains (adcx / adox), then the
 * reduction in two steps.  p = 1 mod 2^192, so M = -t[0..2] mod 2^192 clears the
 * three low limbs at once: t + M p = t + M + (M * 0x0800000000000011) 2^192, the
 * three 64 x 64 products of M * p3 independent of one another; then the usual
 * word step m = -t3 clears limb 3.  This is the same Montgomery quotient as the
 * word-by-word form (the unique m < 2^256 with t + m p = 0 mod 2^256), with a
 * shorter dependency chain.  The result is < 2p and is reduced once with cmov.
 *
 * void zk_felt_mont_cube_adx(uint64_t r[4], const uint64_t a[4]);
 *   r = a^3 / R^2 mod p (two multiplications without a second call), for a < 5p, left
 *   unreduced: the product (a < 5p) * (b < 5p) / R is below p + 25 p^2 / 2^256 < 1.8 p, so a^2 is
 *   below 1.8 p and a^3 below 1.3 p; skipping the final conditional subtraction takes it off the
 *   S-box's latency chain.
 */
/* (rdi) = (rsi) * (rcx) / R mod p; clobbers rax, rbx, rcx, rbp, rdx, r8-r15; keeps rdi, rsi */
.macro MONT_ROWS
    /* row 0: t[0..4] = a * b0 */
    movq    (%rcx), %rdx
    mulxq   (%rsi), %r8, %r9
    mulxq   8(%rsi), %rax, %r10
    addq    %rax, %r9
    mulxq   16(%rsi), %rax, %r11
    adcq    %rax, %r10
    mulxq   24(%rsi), %rax, %r12
    adcq    %rax, %r11
    adcq    $0, %r12

    /* row 1: t[1..5] += a * b1 */
    movq    8(%rcx), %rdx
    xorl    %ebp, %ebp
    mulxq   (%rsi), %rax, %rbx
    adcxq   %rax, %r9
    adoxq   %rbx, %r10
    mulxq   8(%rsi), %rax, %rbx
    adcxq   %rax, %r10
    adoxq   %rbx, %r11
    mulxq   16(%rsi), %rax, %rbx
    adcxq   %rax, %r11
    adoxq   %rbx, %r12
    mulxq   24(%rsi), %rax, %r13
    adcxq   %rax, %r12
    adoxq   %rbp, %r13
    adcxq   %rbp, %r13

    /* row 2: t[2..6] += a * b2 */
    movq    16(%rcx), %rdx
    xorl    %ebp, %ebp
    mulxq   (%rsi), %rax, %rbx
    adcxq   %rax, %r10
    adoxq   %rbx, %r11
    mulxq   8(%rsi), %rax, %rbx
    adcxq   %rax, %r11
    adoxq   %rbx, %r12
    mulxq   16(%rsi), %rax, %rbx
    adcxq   %rax, %r12
    adoxq   %rbx, %r13
    mulxq   24(%rsi), %rax, %r14
    adcxq   %rax, %r13
    adoxq   %rbp, %r14
    adcxq   %rbp, %r14

    /* row 3: t[3..7] += a * b3 */
    movq    24(%rcx), %rdx
    xorl    %ebp, %ebp
    mulxq   (%rsi), %rax, %rbx
    adcxq   %rax, %r11
    adoxq   %rbx, %r12
    mulxq   8(%rsi), %rax, %rbx
    adcxq   %rax, %r12
    adoxq   %rbx, %r13
    mulxq   16(%rsi), %rax, %rbx
    adcxq   %rax, %r13
    adoxq   %rbx, %r14
    mulxq   24(%rsi), %rax, %r15
    adcxq   %rax, %r14
    adoxq   %rbp, %r15
    adcxq   %rbp, %r15

.endm

/* (rdi) = t[0..7] (r8-r15) / R mod p, reduced below p when reduce=1; clobbers rax, rbx, rcx, rbp,
 * rdx, r8-r15 */
.macro MONT_REDUCE reduce=1
    /* reduction step 1: M = -t[0..2] mod 2^192 in rax, rbx, rbp; CF: t[0..2] != 0 */
    xorl    %eax, %eax
    xorl    %ebx, %ebx
    xorl    %ebp, %ebp
    subq    %r8, %rax
    sbbq    %r9, %rbx
    sbbq    %r10, %rbp
    movq    %r8, %rcx                   /* rcx = t[0] | t[1] | t[2] (b is no longer needed) */
    orq     %r9, %rcx
    orq     %r10, %rcx
    /* t[3..7] += M * p3, and the carry of t[0..2] + M (set iff t[0..2] != 0) enters with the
     * first addition instead of rippling through its own chain */
    movabsq $0x0800000000000011, %rdx
    mulxq   %rax, %r8, %r9
    mulxq   %rbx, %r10, %rax
    mulxq   %rbp, %rbx, %rbp
    negq    %rcx
    adcq    %r8, %r11
    adcq    %r9, %r12
    adcq    %rax, %r13
    adcq    %rbp, %r14
    adcq    $0, %r15
    addq    %r10, %r12
    adcq    %rbx, %r13
    adcq    $0, %r14
    adcq    $0, %r15
    /* reduction step 2: m = -t3 clears limb 3, m * p3 lands on limbs 6, 7 */
    movq    %r11, %rdx
    negq    %rdx                        /* CF: t3 != 0 (mov and mulx keep the flags) */
    movabsq $0x0800000000000011, %r8
    mulxq   %r8, %rax, %rbx
    adcq    $0, %r12
    adcq    $0, %r13
    adcq    %rax, %r14
    adcq    %rbx, %r15
    .if \reduce
    /* r = t[4..7] - p if t >= p (branch-free) */
    movq    %r12, %rax
    subq    $1, %rax
    movq    %r13, %rbx
    sbbq    $0, %rbx
    movq    %r14, %rdx
    sbbq    $0, %rdx
    movq    %r15, %rbp
    sbbq    %r8, %rbp
    cmovncq %rax, %r12
    cmovncq %rbx, %r13
    cmovncq %rdx, %r14
    cmovncq %rbp, %r15
    .endif
    movq    %r12, (%rdi)
    movq    %r13, 8(%rdi)
    movq    %r14, 16(%rdi)
    movq    %r15, 24(%rdi)
.endm

/* (rdi) = (rsi) * (rcx) / R mod p; clobbers rax, rbx, rcx, rbp, rdx, r8-r15; keeps rdi, rsi */
.macro MONT_MUL reduce=1
    MONT_ROWS
    MONT_REDUCE \reduce
.endm

/* t[0..7] (r8-r15) = (rsi)^2: the six cross products once, doubled with one shift chain, then
 * the four squares on the diagonal; mov and mulx leave the flags, so the final carry chain runs
 * through the diagonal products as they arrive.  Clobbers rax, rbx, rcx, rdx. */
.macro SQR_ROWS
    movq    (%rsi), %rdx
    mulxq   8(%rsi), %r9, %r10          /* a0 a1 -> t1, t2 */
    mulxq   16(%rsi), %rax, %r11        /* a0 a2 -> t2, t3 */
    addq    %rax, %r10
    mulxq   24(%rsi), %rax, %r12        /* a0 a3 -> t3, t4 */
    adcq    %rax, %r11
    adcq    $0, %r12
    movq    8(%rsi), %rdx
    mulxq   16(%rsi), %rax, %rbx        /* a1 a2 -> t3, t4 */
    mulxq   24(%rsi), %rcx, %r13        /* a1 a3 -> t4, t5 */
    addq    %rax, %r11
    adcq    %rbx, %r12
    adcq    $0, %r13
    addq    %rcx, %r12
    adcq    $0, %r13
    movq    16(%rsi), %rdx
    mulxq   24(%rsi), %rax, %r14        /* a2 a3 -> t5, t6 */
    addq    %rax, %r13
    adcq    $0, %r14
    /* double t1..t6 into t1..t7 */
    xorl    %r15d, %r15d
    shldq   $1, %r14, %r15
    shldq   $1, %r13, %r14
    shldq   $1, %r12, %r13
    shldq   $1, %r11, %r12
    shldq   $1, %r10, %r11
    shldq   $1, %r9, %r10
    addq    %r9, %r9
    /* + a_i^2 at t[2i], t[2i+1] */
    movq    (%rsi), %rdx
    mulxq   %rdx, %r8, %rax
    movq    8(%rsi), %rdx
    mulxq   %rdx, %rbx, %rcx
    addq    %rax, %r9
    adcq    %rbx, %r10
    adcq    %rcx, %r11
    movq    16(%rsi), %rdx
    mulxq   %rdx, %rax, %rbx
    adcq    %rax, %r12
    adcq    %rbx, %r13
    movq    24(%rsi), %rdx
    mulxq   %rdx, %rax, %rbx
    adcq    %rax, %r14
    adcq    %rbx, %r15
.endm

    .text
    .globl  zk_felt_mont_mul_adx
    .type   zk_felt_mont_mul_adx, @function
    .p2align 4
zk_felt_mont_mul_adx:
    pushq   %rbx
    pushq   %rbp
    pushq   %r12
    pushq   %r13
    pushq   %r14
    pushq   %r15
    movq    %rdx, %rcx                  /* rcx = b */
    MONT_MUL
    popq    %r15
    popq    %r14
    popq    %r13
    popq    %r12
    popq    %rbp
    popq    %rbx
    ret
    .size   zk_felt_mont_mul_adx, .-zk_felt_mont_mul_adx

    .globl  zk_felt_mont_cube_adx
    .type   zk_felt_mont_cube_adx, @function
    .p2align 4
zk_felt_mont_cube_adx:
    pushq   %rbx
    pushq   %rbp
    pushq   %r12
    pushq   %r13
    pushq   %r14
    pushq   %r15
    subq    $40, %rsp
    movq    %rdi, 32(%rsp)              /* the result pointer */
    movq    %rsp, %rdi                  /* a^2 into the stack slot, left below 1.8 p (not reduced) */
    SQR_ROWS
    MONT_REDUCE 0
    movq    %rsp, %rcx                  /* b = a^2 */
    movq    32(%rsp), %rdi
    MONT_MUL 0                          /* a^3 below 1.3 p (not reduced) */
    addq    $40, %rsp
    popq    %r15
    popq    %r14
    popq    %r13
    popq    %r12
    popq    %rbp
    popq    %rbx
    ret
    .size   zk_felt_mont_cube_adx, .-zk_felt_mont_cube_adx
    .section .note.GNU-stack,"",@progbits
