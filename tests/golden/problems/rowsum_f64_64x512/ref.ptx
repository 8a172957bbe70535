.version 8.0
.target sm_89
.address_size 64

.shared .align 8 .b8 red_smem[32];

.visible .entry k_rowsum_f64(
        .param .u64 p_x,
        .param .u64 p_out
)
{
        .reg .pred %p<7>;
        .reg .f32  %f<1>;
        .reg .b16  %h<1>;
        .reg .f64  %d<14>;
        .reg .b32  %r<66>;
        .reg .b64  %rd<27>;

        ld.param.u64 %rd1, [p_x];
        cvta.to.global.u64 %rd2, %rd1;
        ld.param.u64 %rd3, [p_out];
        cvta.to.global.u64 %rd4, %rd3;
        mov.u32 %r1, %tid.x;
        and.b32 %r2, %r1, 31;
        shr.u32 %r3, %r1, 5;
        mov.u32 %r4, red_smem;
        mov.u32 %r5, %ctaid.x;
        mad.lo.u32 %r6, %r5, 128, %r1;
        setp.ge.u32 %p1, %r6, 8192;
        @%p1 bra TILE_END_1;
        div.s32 %r7, %r6, 128;
        rem.s32 %r8, %r6, 128;
        mov.u32 %r9, 0x00000000;
        mov.u32 %r10, 0x00000000;
        mov.b64 %rd5, {%r9, %r10};
        mov.f64 %d1, %rd5;
        mov.s32 %r11, %r8;
        mov.s32 %r12, 128;
        mov.s32 %r13, 256;
SL_2:
        setp.ge.s32 %p2, %r11, %r13;
        @%p2 bra SL_END_3;
        mul.lo.s32 %r14, %r7, 512;
        mov.s32 %r15, 2;
        mul.lo.s32 %r16, %r11, %r15;
        add.s32 %r17, %r14, %r16;
        mul.wide.s32 %rd6, %r17, 8;
        add.s64 %rd7, %rd2, %rd6;
        ld.global.f64 %d2, [%rd7];
        mul.lo.s32 %r18, %r7, 512;
        mov.s32 %r19, 2;
        mul.lo.s32 %r20, %r11, %r19;
        mov.s32 %r21, 1;
        add.s32 %r22, %r20, %r21;
        add.s32 %r23, %r18, %r22;
        mul.wide.s32 %rd8, %r23, 8;
        add.s64 %rd9, %rd2, %rd8;
        ld.global.f64 %d3, [%rd9];
        add.f64 %d1, %d1, %d2;
        add.f64 %d1, %d1, %d3;
        add.s32 %r11, %r11, %r12;
        bra SL_2;
SL_END_3:
        activemask.b32 %r24;
        mov.b64 %rd10, %d1;
        cvt.u32.u64 %r25, %rd10;
        shr.u64 %rd11, %rd10, 32;
        cvt.u32.u64 %r26, %rd11;
        shfl.sync.bfly.b32 %r27, %r25, 16, 0x1f, %r24;
        shfl.sync.bfly.b32 %r28, %r26, 16, 0x1f, %r24;
        mov.b64 %rd12, {%r27, %r28};
        mov.f64 %d4, %rd12;
        add.f64 %d1, %d1, %d4;
        mov.b64 %rd13, %d1;
        cvt.u32.u64 %r29, %rd13;
        shr.u64 %rd14, %rd13, 32;
        cvt.u32.u64 %r30, %rd14;
        shfl.sync.bfly.b32 %r31, %r29, 8, 0x1f, %r24;
        shfl.sync.bfly.b32 %r32, %r30, 8, 0x1f, %r24;
        mov.b64 %rd15, {%r31, %r32};
        mov.f64 %d5, %rd15;
        add.f64 %d1, %d1, %d5;
        mov.b64 %rd16, %d1;
        cvt.u32.u64 %r33, %rd16;
        shr.u64 %rd17, %rd16, 32;
        cvt.u32.u64 %r34, %rd17;
        shfl.sync.bfly.b32 %r35, %r33, 4, 0x1f, %r24;
        shfl.sync.bfly.b32 %r36, %r34, 4, 0x1f, %r24;
        mov.b64 %rd18, {%r35, %r36};
        mov.f64 %d6, %rd18;
        add.f64 %d1, %d1, %d6;
        mov.b64 %rd19, %d1;
        cvt.u32.u64 %r37, %rd19;
        shr.u64 %rd20, %rd19, 32;
        cvt.u32.u64 %r38, %rd20;
        shfl.sync.bfly.b32 %r39, %r37, 2, 0x1f, %r24;
        shfl.sync.bfly.b32 %r40, %r38, 2, 0x1f, %r24;
        mov.b64 %rd21, {%r39, %r40};
        mov.f64 %d7, %rd21;
        add.f64 %d1, %d1, %d7;
        mov.b64 %rd22, %d1;
        cvt.u32.u64 %r41, %rd22;
        shr.u64 %rd23, %rd22, 32;
        cvt.u32.u64 %r42, %rd23;
        shfl.sync.bfly.b32 %r43, %r41, 1, 0x1f, %r24;
        shfl.sync.bfly.b32 %r44, %r42, 1, 0x1f, %r24;
        mov.b64 %rd24, {%r43, %r44};
        mov.f64 %d8, %rd24;
        add.f64 %d1, %d1, %d8;
        mov.s32 %r45, 0;
        setp.eq.s32 %p3, %r2, %r45;
        @!%p3 bra ELSE_4;
        mul.lo.s32 %r46, %r3, 8;
        add.s32 %r47, %r4, %r46;
        st.shared.f64 [%r47], %d1;
        bra COND_END_5;
ELSE_4:
COND_END_5:
        bar.sync 0;
        setp.lt.s32 %p4, %r8, 2;
        @!%p4 bra TREE_SKIP_6;
        add.s32 %r48, %r8, 2;
        mul.lo.s32 %r49, %r8, 8;
        add.s32 %r50, %r4, %r49;
        mul.lo.s32 %r51, %r48, 8;
        add.s32 %r52, %r4, %r51;
        ld.shared.f64 %d9, [%r50];
        ld.shared.f64 %d10, [%r52];
        add.f64 %d9, %d9, %d10;
        mul.lo.s32 %r53, %r8, 8;
        add.s32 %r54, %r4, %r53;
        st.shared.f64 [%r54], %d9;
TREE_SKIP_6:
        bar.sync 0;
        setp.lt.s32 %p5, %r8, 1;
        @!%p5 bra TREE_SKIP_7;
        add.s32 %r55, %r8, 1;
        mul.lo.s32 %r56, %r8, 8;
        add.s32 %r57, %r4, %r56;
        mul.lo.s32 %r58, %r55, 8;
        add.s32 %r59, %r4, %r58;
        ld.shared.f64 %d11, [%r57];
        ld.shared.f64 %d12, [%r59];
        add.f64 %d11, %d11, %d12;
        mul.lo.s32 %r60, %r8, 8;
        add.s32 %r61, %r4, %r60;
        st.shared.f64 [%r61], %d11;
TREE_SKIP_7:
        bar.sync 0;
        mov.s32 %r62, 0;
        mul.lo.s32 %r63, %r62, 8;
        add.s32 %r64, %r4, %r63;
        ld.shared.f64 %d13, [%r64];
        mov.s32 %r65, 0;
        setp.eq.s32 %p6, %r8, %r65;
        @!%p6 bra ELSE_8;
        mul.wide.s32 %rd25, %r7, 8;
        add.s64 %rd26, %rd4, %rd25;
        st.global.f64 [%rd26], %d13;
        bra COND_END_9;
ELSE_8:
COND_END_9:
TILE_END_1:
        ret;
}
